// Host harness for the step kernel's plan (test infrastructure, no GPU):
// reads model shapes from stdin, one per line,
//   n_layers dim n_heads n_kv_heads head_dim ffn vocab t_embd t_qkv t_o t_gu t_down t_out tp n_sm
// and prints the plan vbs::step_plan makes for each as one JSON line.
// tests/test_step_plan.py compiles it together with the library's step.cu.
#include "common.cuh"
#include "kernels.h"

#include <cstdio>

namespace vbs {
void note_launches(unsigned long) {}   // the launch counter lives in backend.cu
}

int main() {
    using namespace vbs;
    static TpComm comm{};   // only its presence matters to the plan
    unsigned L, dim, nqh, nkh, hd, ffn, vocab, tp, n_sm;
    int te, tq, to, tg, td, tout;
    while (scanf("%u %u %u %u %u %u %u %d %d %d %d %d %d %u %u", &L, &dim, &nqh, &nkh, &hd, &ffn, &vocab, &te, &tq, &to, &tg,
                 &td, &tout, &tp, &n_sm) == 15) {
        StepParams p{};
        p.n_layers = L; p.dim = dim; p.nqh = nqh; p.nkh = nkh; p.hd = hd; p.ffn = ffn; p.vocab = vocab;
        p.max_ctx = 8192;
        p.t_embd = te; p.t_qkv = tq; p.t_o = to; p.t_gu = tg; p.t_down = td; p.t_out = tout;
        p.tp = tp ? &comm : nullptr;
        char why[160] = "";
        const bool ok = step_plan(p, (int)n_sm, why, sizeof why);
        printf("{\"ok\": %d, \"why\": \"%s\", \"geo\": [", ok ? 1 : 0, why);
        for (int k = 0; k < 5; ++k)
            printf("%s[%u, %u, %u, %u]", k ? ", " : "", p.geo[k].ck, p.geo[k].rs, p.geo[k].nch, p.geo[k].ntiles);
        printf("], \"x_off\": %u, \"xq_off\": %u, \"xf_off\": %u, \"ring_off\": %u, \"ring_bytes\": %u, \"stage_max\": %u, "
               "\"attn_splits\": %u, \"acc_layer\": %llu}\n",
               p.x_off, p.xq_off, p.xf_off, p.ring_off, p.ring_bytes, p.stage_max, p.attn_splits,
               (unsigned long long)p.acc_layer);
    }
    return 0;
}
