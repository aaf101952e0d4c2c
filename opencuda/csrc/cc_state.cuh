// Per-TU state kept at the start of the TU's arena slice between the
// compiler's kernels (parse -> optimize -> emit): the two arenas and the IR.
#pragma once
#include "cc_ir.cuh"

namespace ocb {
namespace cc {

enum { CC_STAGE_IR = 0, CC_STAGE_OPT = 1, CC_STAGE_PTX = 2 };

// Minimum resident 128-thread blocks per SM requested from the compiler for
// the parse/optimize/emit kernels (caps their registers per thread).  The
// parser and the emitter run faster at 80 registers (six blocks, 24 warps per
// SM) despite a few spills; the optimizer's pass loops keep their registers.
#ifndef OCB_CC_MIN_BLOCKS
#define OCB_CC_MIN_BLOCKS 1
#endif
#ifndef OCB_CC_MIN_BLOCKS_PARSE
#define OCB_CC_MIN_BLOCKS_PARSE 6
#endif
#ifndef OCB_CC_MIN_BLOCKS_OPT
#define OCB_CC_MIN_BLOCKS_OPT OCB_CC_MIN_BLOCKS
#endif
#ifndef OCB_CC_MIN_BLOCKS_EMIT
#define OCB_CC_MIN_BLOCKS_EMIT 6
#endif

struct TUState {
    Arena ar;    // the IR (3/4 of the slice after this header)
    Arena tmp;   // per-pass scratch (1/4)
    Module m;
    int32_t status;  // OCB_TU_* (0 = carry on)
};

struct CCArgs {
    const uint8_t *src;          // preprocessed text of the batch
    const uint32_t *tok_start;   // token starts (batch offsets)
    const uint32_t *tok_kl;      // kind << 24 | length
    const uint64_t *tu_tok_off;  // n_tu + 1
    uint32_t n_tu;
    uint8_t *arena;
    const uint64_t *arena_off;
    uint8_t *out;
    const uint64_t *out_off;     // capacity offsets
    uint64_t *out_len;           // n_tu + 1 (last = 0)
    int32_t *status;             // in: earlier stages' verdicts; out: final
    int stage;
    uint32_t spread;             // TUs per warp (1..32): lane < spread works
    uint32_t ir_permille;        // share of a TU's slice for the IR (rest: scratch)
    uint64_t *peak;              // optional: per-TU arena bytes used (tuning)
    char target[32];             // `.target` of the module header (NUL terminated)
    const uint32_t *order;       // optional: TU of each thread slot (largest first)
    SpillPool spill;             // shared overflow space of this launch
};

// TU index of this thread, or n_tu when the lane is idle
OCB_HD inline uint32_t cc_tu_index(const CCArgs &A) {
#ifdef __CUDA_ARCH__
    uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t lane = g & 31, warp = g >> 5;
    if (lane >= A.spread) return 0xFFFFFFFFu;
    uint32_t j = warp * A.spread + lane;
    if (j >= A.n_tu) return 0xFFFFFFFFu;
    return A.order ? A.order[j] : j;
#else
    return 0xFFFFFFFFu;
#endif
}

OCB_HD inline TUState *tu_state(const CCArgs &A, uint32_t i) {
    return (TUState *)(A.arena + A.arena_off[i]);
}

}  // namespace cc
}  // namespace ocb
