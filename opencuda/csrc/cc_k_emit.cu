// Compiler kernel 3 of 3: write each TU's output text -- the PTX module
// (stage PTX) or the IR in canonical text (stages IR / OPT).
#include <cuda_runtime.h>
#include "../../include/ocb.h"
#include "cc_state.cuh"
#include "cc_emit_kernel.cuh"
#include "cc_dump.cuh"

namespace ocb {
namespace cc {

__global__ void __launch_bounds__(128, OCB_CC_MIN_BLOCKS_EMIT) k_cc_emit(CCArgs A) {
    uint32_t i = cc_tu_index(A);
    if (i >= A.n_tu) return;
    A.out_len[i] = 0;
    if (A.status[i] != 0) return;
    TUState *S = tu_state(A, i);
    Module &m = S->m;
    m.ar = &S->ar;
    Out o{(char *)A.out + A.out_off[i], 0, A.out_off[i + 1] - A.out_off[i], false};
    int32_t st = OCB_TU_OK;
    if (A.stage >= CC_STAGE_PTX) {
        S->tmp.used = 0;
        bool ok = emit_module(m, S->tmp, o, A.target);
        if (S->ar.oom || S->tmp.oom || o.full) st = OCB_TU_OVERFLOW;
        else if (m.unsup || (!ok && !m.raises)) st = OCB_TU_UNSUPPORTED;
        else if (!ok) st = m.raises;
    } else {
        dump_module(o, m);
        if (o.full) st = OCB_TU_OVERFLOW;
    }
    A.status[i] = st;
    if (st == OCB_TU_OK) A.out_len[i] = o.n;
    if (A.peak) A.peak[i] = S->ar.used;
}

// host-side launcher (kernels of separate objects are launched from here)
cudaError_t launch_k_cc_emit(const CCArgs &A, unsigned grid, unsigned block, cudaStream_t st) {
    k_cc_emit<<<grid, block, 0, st>>>(A);
    return cudaGetLastError();
}

// the kernel's entry, for function attributes set by the driver code
const void *k_cc_emit_entry() { return (const void *)k_cc_emit; }

}  // namespace cc
}  // namespace ocb
