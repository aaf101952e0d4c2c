// Batch compiler back half for sm_100a: tokens -> IR (-> PTX), one thread per
// translation unit.  Each TU gets a private slice of one arena buffer sized
// from its token count; a TU that outgrows it reports OCB_TU_OVERFLOW and the
// host runs it again with a larger slice.
#include <cub/cub.cuh>
#include "ocb_internal.h"
#include "cc_state.cuh"

namespace ocb {
namespace cc {

cudaError_t launch_k_cc_parse(const CCArgs &A, unsigned grid, unsigned block, cudaStream_t st);
cudaError_t launch_k_cc_opt(const CCArgs &A, unsigned grid, unsigned block, cudaStream_t st);
cudaError_t launch_k_cc_emit(const CCArgs &A, unsigned grid, unsigned block, cudaStream_t st);

// Per-TU arena and output sizes (bytes, 16-aligned) from the token counts.
__global__ void k_cc_sizes(const uint64_t *tu_tok_off, uint32_t n_tu, uint32_t scale,
                           uint64_t *arena_sz, uint64_t *out_sz) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i > n_tu) return;
    if (i == n_tu) {
        arena_sz[i] = 0;
        out_sz[i] = 0;
        return;
    }
    uint64_t nt = tu_tok_off[i + 1] - tu_tok_off[i];
    arena_sz[i] = ((65536ull + 2048ull * nt) * scale + 15) & ~15ull;
    out_sz[i] = ((4096ull + 256ull * nt) * scale + 15) & ~15ull;
}

__global__ void merge_status(int32_t *st, const int32_t *lex_st, uint32_t n_tu) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_tu && st[i] == 0 && lex_st[i] != 0) st[i] = lex_st[i];
}

// Gather each TU's output into one packed buffer; one block per TU.
__global__ void k_cc_pack(const uint8_t *out, const uint64_t *cap_off, const uint64_t *pack_off,
                          uint8_t *dst, uint32_t n_tu) {
    uint32_t i = blockIdx.x;
    if (i >= n_tu) return;
    const uint8_t *s = out + cap_off[i];
    uint8_t *d = dst + pack_off[i];
    uint64_t n = pack_off[i + 1] - pack_off[i];
    for (uint64_t k = threadIdx.x; k < n; k += blockDim.x) d[k] = s[k];
}

}  // namespace cc

// Device stack for the recursive-descent parser: frames are bounded by
// cc::MAX_NEST (expression and statement nesting).
static constexpr size_t kCCStack = 64 * 1024;

int cc_device(ocb_ctx *ctx, const uint8_t *d_text, uint64_t N, const uint64_t *d_off,
              uint32_t n_tu, const int32_t *d_in_status, int stage, uint32_t scale,
              DevBuf &out_text, uint64_t *d_out_off, int32_t *d_status, uint64_t *h_total,
              cudaStream_t st) {
    using namespace cc;
    if (n_tu == 0) {
        *h_total = 0;
        OCB_TRY("cc: zero TUs", cudaMemsetAsync(d_out_off, 0, 8, st));
        return 0;
    }
    size_t n1 = (size_t)n_tu + 1;
    uint64_t tok_cap = N + n_tu + 16;
    OCB_TRY("cc: tokens", ctx->cc_tok.ensure(12 * tok_cap + 16));
    OCB_TRY("cc: scratch", ctx->cc_scratch.ensure(8 * n1 * 7 + 4 * n1 + 64));
    uint32_t *tstart = ctx->cc_tok.as<uint32_t>();
    uint32_t *tkl = tstart + tok_cap;
    uint32_t *tline = tkl + tok_cap;
    uint64_t *tu_tok = ctx->cc_scratch.as<uint64_t>();
    uint64_t *arena_sz = tu_tok + n1;
    uint64_t *arena_off = arena_sz + n1;
    uint64_t *out_sz = arena_off + n1;
    uint64_t *out_cap_off = out_sz + n1;
    uint64_t *out_len = out_cap_off + n1;
    uint64_t *n_tok = out_len + n1;
    int32_t *lex_status = (int32_t *)(n_tok + 1);
    int rc = lex_device(ctx, d_text, N, d_off, n_tu, tstart, tkl, tline, tok_cap, tu_tok,
                        lex_status, n_tok, st);
    if (rc) return rc;
    // merged status of preprocessing and lexing feeds the parser
    OCB_TRY("cc: status", cudaMemcpyAsync(d_status, d_in_status, 4 * (size_t)n_tu,
                                          cudaMemcpyDeviceToDevice, st));
    size_t t1 = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, t1, arena_sz, arena_off, (int)n1, st);
    OCB_TRY("cc: cub scratch", ctx->cub_tmp.ensure(t1));
    unsigned grid = (unsigned)((n1 + 255) / 256);
    k_cc_sizes<<<grid, 256, 0, st>>>(tu_tok, n_tu, scale, arena_sz, out_sz);
    OCB_TRY("cc: arena scan",
            cub::DeviceScan::ExclusiveSum(ctx->cub_tmp.p, t1, arena_sz, arena_off, (int)n1, st));
    OCB_TRY("cc: out scan",
            cub::DeviceScan::ExclusiveSum(ctx->cub_tmp.p, t1, out_sz, out_cap_off, (int)n1, st));
    uint64_t tot[2] = {0, 0};
    OCB_TRY("cc: d2h", cudaMemcpyAsync(&tot[0], arena_off + n_tu, 8, cudaMemcpyDeviceToHost, st));
    OCB_TRY("cc: d2h", cudaMemcpyAsync(&tot[1], out_cap_off + n_tu, 8, cudaMemcpyDeviceToHost, st));
    OCB_TRY("cc: sync", cudaStreamSynchronize(st));
    OCB_TRY("cc: arena", ctx->cc_arena.ensure(tot[0] + 64));
    OCB_TRY("cc: out", ctx->cc_out.ensure(tot[1] + 64));
    // lexer verdicts (hex-float ValueError / OverflowError) stop a TU before parsing
    merge_status<<<grid, 256, 0, st>>>(d_status, lex_status, n_tu);
    size_t cur_stack = 0;
    OCB_TRY("cc: stack limit", cudaDeviceGetLimit(&cur_stack, cudaLimitStackSize));
    if (cur_stack < kCCStack) OCB_TRY("cc: stack limit", cudaDeviceSetLimit(cudaLimitStackSize, kCCStack));
    CCArgs A{d_text, tstart, tkl, tu_tok, n_tu, ctx->cc_arena.as<uint8_t>(), arena_off,
             ctx->cc_out.as<uint8_t>(), out_cap_off, out_len, d_status, stage};
    unsigned g64 = (unsigned)((n1 + 63) / 64);
    OCB_TRY("cc: parse launch", launch_k_cc_parse(A, g64, 64, st));
    if (stage >= CC_STAGE_OPT) OCB_TRY("cc: optimize launch", launch_k_cc_opt(A, g64, 64, st));
    OCB_TRY("cc: emit launch", launch_k_cc_emit(A, g64, 64, st));
    OCB_TRY("cc: pack scan",
            cub::DeviceScan::ExclusiveSum(ctx->cub_tmp.p, t1, out_len, d_out_off, (int)n1, st));
    uint64_t total = 0;
    OCB_TRY("cc: d2h", cudaMemcpyAsync(&total, d_out_off + n_tu, 8, cudaMemcpyDeviceToHost, st));
    OCB_TRY("cc: sync", cudaStreamSynchronize(st));
    OCB_TRY("cc: output", out_text.ensure(total + 64));
    k_cc_pack<<<n_tu, 128, 0, st>>>(ctx->cc_out.as<uint8_t>(), out_cap_off, d_out_off,
                                    out_text.as<uint8_t>(), n_tu);
    OCB_TRY("cc: pack launch", cudaGetLastError());
    *h_total = total;
    return 0;
}

}  // namespace ocb
