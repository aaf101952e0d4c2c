// Compiler kernel for the IR verifier stages: check each TU's IR (after
// parse, or after optimize) with the invariants of opencuda/ir/verify_ir.py
// and write the error text (cc_verify.cuh).  Launched in place of the emit
// kernel.
#include <cuda_runtime.h>
#include "../../include/ocb.h"
#include "cc_state.cuh"
#include "cc_verify.cuh"

namespace ocb {
namespace cc {

__global__ void __launch_bounds__(128, OCB_CC_MIN_BLOCKS) k_cc_verify(CCArgs A, int check_reach) {
    uint32_t i = cc_tu_index(A);
    if (i >= A.n_tu) return;
    A.out_len[i] = 0;
    if (A.status[i] != 0) return;
    TUState *S = tu_state(A, i);
    Module &m = S->m;
    m.ar = &S->ar;
    Out o{(char *)A.out + A.out_off[i], 0, A.out_off[i + 1] - A.out_off[i], false};
    S->tmp.used = 0;
    bool ok = verify_module(m, S->tmp, o, check_reach != 0);
    int32_t st = OCB_TU_OK;
    if (S->ar.oom || S->tmp.oom || o.full) st = OCB_TU_OVERFLOW;
    else if (!ok) st = OCB_TU_UNSUPPORTED;
    A.status[i] = st;
    if (st == OCB_TU_OK) A.out_len[i] = o.n;
}

cudaError_t launch_k_cc_verify(const CCArgs &A, int check_reach, unsigned grid, unsigned block,
                               cudaStream_t st) {
    k_cc_verify<<<grid, block, 0, st>>>(A, check_reach);
    return cudaGetLastError();
}

}  // namespace cc
}  // namespace ocb
