// upload.cu -- byte ranges of a file straight into device memory.
//
// The reference loads a model by keeping every tensor in a host mirror and
// calling the backend's copy_to_device once per tensor, synchronously
// (src/vbs_fabric.c:81-94 through src/vbs_backend_cuda.c:148). Here the
// caller hands over all ranges at once. Reader threads pread chunks of the
// file into pinned staging buffers, two per thread, and copy each chunk
// with cudaMemcpyAsync on the thread's own stream while they read the next
// one. File reads (disk or page cache) and host-to-device copies overlap,
// and no host copy of the model is ever held. Host code only.
#include "vbs_b200.h"
#include "backend.h"

#include <cerrno>
#include <cstring>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

struct Chunk {
    uint64_t off, len;   // file range
    uint8_t *dst;        // device destination of its first byte
};

struct Upload {
    std::vector<Chunk> chunks;
    std::atomic<size_t> next{0};
    std::atomic<bool> failed{false};
    std::mutex mu;
    std::string err;
    int fd = -1, device = 0;
    uint64_t chunk_bytes = 0;

    void fail(const std::string &m) {
        std::lock_guard<std::mutex> g(mu);
        if (err.empty()) err = m;
        failed = true;
    }
    bool cuda(cudaError_t e, const char *what) {
        if (e == cudaSuccess) return true;
        fail(std::string(what) + ": " + cudaGetErrorString(e));
        return false;
    }
};

// One reader thread: chunks in the order the shared counter hands them out;
// buffer b is reused only after the copy that last read it has finished.
void reader(Upload *u) {
    if (!u->cuda(cudaSetDevice(u->device), "cudaSetDevice")) return;
    cudaStream_t st = nullptr;
    uint8_t *buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool busy[2] = {false, false};
    bool ok = u->cuda(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking), "upload stream");
    for (int i = 0; i < 2 && ok; ++i)
        ok = u->cuda(cudaHostAlloc(reinterpret_cast<void **>(&buf[i]), u->chunk_bytes, cudaHostAllocDefault),
                     "pinned staging buffer") &&
             u->cuda(cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming), "upload event");
    for (int b = 0; ok && !u->failed;) {
        const size_t i = u->next.fetch_add(1);
        if (i >= u->chunks.size()) break;
        const Chunk &c = u->chunks[i];
        if (busy[b] && !u->cuda(cudaEventSynchronize(ev[b]), "upload copy")) break;
        for (uint64_t got = 0; got < c.len;) {
            const ssize_t r = pread(u->fd, buf[b] + got, c.len - got, static_cast<off_t>(c.off + got));
            if (r < 0 && errno == EINTR) continue;
            if (r <= 0) {
                u->fail(r == 0 ? std::string("file ended early") : std::string("read: ") + strerror(errno));
                break;
            }
            got += static_cast<uint64_t>(r);
        }
        if (u->failed) break;
        if (!u->cuda(cudaMemcpyAsync(c.dst, buf[b], c.len, cudaMemcpyHostToDevice, st), "cudaMemcpyAsync") ||
            !u->cuda(cudaEventRecord(ev[b], st), "upload event"))
            break;
        busy[b] = true;
        b ^= 1;
    }
    if (st) u->cuda(cudaStreamSynchronize(st), "upload copy");
    for (int i = 0; i < 2; ++i) {
        if (ev[i]) cudaEventDestroy(ev[i]);
        if (buf[i]) cudaFreeHost(buf[i]);
    }
    if (st) cudaStreamDestroy(st);
}

}  // namespace

using namespace vbs;

extern "C" {

int vbs_cu_upload_file(const char *path, size_t n, const uint64_t *offsets, const uint64_t *sizes, void *const *dst,
                       uint32_t n_threads, uint64_t chunk_bytes) {
    if (!path || (n && (!offsets || !sizes || !dst))) { latch_error("upload_file: invalid arguments"); return -1; }
    if (!backend_current()) { latch_error("upload_file: no usable device"); return -1; }
    Upload u;
    if (!u.cuda(cudaGetDevice(&u.device), "cudaGetDevice")) { latch_error("upload_file: %s", u.err.c_str()); return -1; }
    u.fd = open(path, O_RDONLY | O_CLOEXEC);
    if (u.fd < 0) { latch_error("upload_file: %s: %s", path, strerror(errno)); return -1; }
    struct stat sb;
    if (fstat(u.fd, &sb) != 0) {
        latch_error("upload_file: %s: %s", path, strerror(errno));
        close(u.fd);
        return -1;
    }
    const uint64_t fsize = static_cast<uint64_t>(sb.st_size);
    u.chunk_bytes = chunk_bytes ? std::min<uint64_t>(std::max<uint64_t>(chunk_bytes, 1ull << 20), 1ull << 30) : 16ull << 20;
    for (size_t i = 0; i < n; ++i) {
        if (offsets[i] > fsize || sizes[i] > fsize - offsets[i]) {
            latch_error("upload_file: range %zu (offset %llu, %llu bytes) is outside the %llu-byte file", i,
                        (unsigned long long)offsets[i], (unsigned long long)sizes[i], (unsigned long long)fsize);
            close(u.fd);
            return -1;
        }
        if (sizes[i] && !dst[i]) { latch_error("upload_file: range %zu has no destination", i); close(u.fd); return -1; }
        for (uint64_t o = 0; o < sizes[i]; o += u.chunk_bytes)
            u.chunks.push_back({offsets[i] + o, std::min(u.chunk_bytes, sizes[i] - o), static_cast<uint8_t *>(dst[i]) + o});
    }
    // largest chunks first, so the threads finish close together
    std::stable_sort(u.chunks.begin(), u.chunks.end(), [](const Chunk &a, const Chunk &b) { return a.len > b.len; });
    const size_t nt = std::min<size_t>(std::max<uint32_t>(1u, std::min<uint32_t>(n_threads ? n_threads : 4u, 32u)),
                                       std::max<size_t>(1, u.chunks.size()));
    if (!u.chunks.empty()) {
        std::vector<std::thread> th;
        th.reserve(nt);
        for (size_t t = 0; t < nt; ++t) th.emplace_back(reader, &u);
        for (std::thread &t : th) t.join();
    }
    close(u.fd);
    if (u.failed) { latch_error("upload_file: %s", u.err.c_str()); return -1; }
    return 0;
}

}  // extern "C"
