// Compiler kernel 1 of 3: parse each TU's tokens into IR (one thread per TU).
#include <new>
#include <cuda_runtime.h>
#include "../../include/ocb.h"
#include "cc_state.cuh"
#include "cc_parse_stmt.cuh"

namespace ocb {
namespace cc {

__global__ void __launch_bounds__(128, OCB_CC_MIN_BLOCKS_PARSE) k_cc_parse(CCArgs A) {
    uint32_t i = cc_tu_index(A);
    if (i >= A.n_tu) return;
    uint64_t sz = A.arena_off[i + 1] - A.arena_off[i];
    TUState *S = tu_state(A, i);
    if (sz < sizeof(TUState) + 4096) {
        A.status[i] = A.status[i] ? A.status[i] : OCB_TU_OVERFLOW;
        return;
    }
    S->status = A.status[i];
    if (S->status != 0) return;
    uint8_t *base = A.arena + A.arena_off[i] + ((sizeof(TUState) + 15) & ~(size_t)15);
    uint64_t rest = sz - ((sizeof(TUState) + 15) & ~(size_t)15);
    uint64_t ir_sz = (rest / 1000 * A.ir_permille) & ~15ull;
    S->ar = Arena{base, 0, ir_sz, false, A.spill};
    S->tmp = Arena{base + ir_sz, 0, rest - ir_sz, false, A.spill};
    S->m.init(&S->ar);
    Parser *P = (Parser *)S->tmp.alloc(sizeof(Parser), 16);
    if (!P) {
        S->status = A.status[i] = OCB_TU_OVERFLOW;
        return;
    }
    uint64_t t0 = A.tu_tok_off[i];
    Tokens t{A.src, A.tok_start + t0, A.tok_kl + t0, (uint32_t)(A.tu_tok_off[i + 1] - t0)};
    // the parser's own tables live in the IR arena; the Parser object in scratch
    new (P) Parser(S->ar, S->m, t);
    P->parse_module();
    int32_t st = 0;
    if (S->ar.oom || S->tmp.oom) st = OCB_TU_OVERFLOW;
    else if (S->m.unsup) st = OCB_TU_UNSUPPORTED;
    else if (P->err) st = S->m.raises;
    S->status = st;
    A.status[i] = st;
}

// host-side launcher (kernels of separate objects are launched from here)
cudaError_t launch_k_cc_parse(const CCArgs &A, unsigned grid, unsigned block, cudaStream_t st) {
    k_cc_parse<<<grid, block, 0, st>>>(A);
    return cudaGetLastError();
}

// the kernel's entry, for function attributes set by the driver code
const void *k_cc_parse_entry() { return (const void *)k_cc_parse; }

}  // namespace cc
}  // namespace ocb
