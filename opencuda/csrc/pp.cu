// Batch preprocessor for sm_100a: host driver (kernels in pp_kernels.cuh).
#include <cub/cub.cuh>
#include "ocb_internal.h"
#include "pp_kernels.cuh"

namespace ocb {

int pp_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t N, const uint64_t *d_tu_off,
              uint32_t n_tu, uint32_t scale, DevBuf &out_text, uint64_t *d_out_off,
              int32_t *d_status, uint32_t *d_qinc, uint64_t *h_total, cudaStream_t st) {
    using namespace pp;
    (void)N;
    if (n_tu == 0) {
        *h_total = 0;
        OCB_TRY("pp: zero TUs", cudaMemsetAsync(d_out_off, 0, 8, st));
        return 0;
    }
    // scratch: arena offsets (n_tu+1), out lengths (n_tu+1 as u64), cub temp
    size_t n1 = (size_t)n_tu + 1;
    OCB_TRY("pp: scratch", ctx->pp_scratch.ensure(8 * n1 * 3 + 4 * n1));
    uint64_t *sizes = ctx->pp_scratch.as<uint64_t>();
    uint64_t *arena_off = sizes + n1;
    uint64_t *len64 = arena_off + n1;
    uint32_t *len32 = (uint32_t *)(len64 + n1);
    size_t t1 = 0, t2 = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, t1, sizes, arena_off, (int)n1, st);
    cub::DeviceScan::ExclusiveSum(nullptr, t2, len64, d_out_off, (int)n1, st);
    OCB_TRY("pp: cub scratch", ctx->cub_tmp.ensure(t1 > t2 ? t1 : t2));
    unsigned grid = (unsigned)((n1 + 255) / 256);
    k_pp_arena_sizes<<<grid, 256, 0, st>>>(d_tu_off, n_tu, scale, sizes);
    OCB_TRY("pp: arena scan",
            cub::DeviceScan::ExclusiveSum(ctx->cub_tmp.p, t1, sizes, arena_off, (int)n1, st));
    uint64_t arena_total = 0;
    OCB_TRY("pp: d2h", cudaMemcpyAsync(&arena_total, arena_off + n_tu, 8, cudaMemcpyDeviceToHost, st));
    OCB_TRY("pp: sync", stream_wait(st));
    OCB_TRY("pp: arena", ctx->pp_arena.ensure(arena_total));
    OCB_TRY("pp: memset", cudaMemsetAsync(d_qinc, 0, 4 * (size_t)n_tu, st));
    PPArgs A{d_src, d_tu_off, n_tu, ctx->pp_arena.as<uint8_t>(), arena_off,
             len32, d_status, d_qinc};
    // one thread per TU; TUs are independent
    k_preprocess<<<(n_tu + 127) / 128, 128, 0, st>>>(A, scale);
    k_widen_u32<<<grid, 256, 0, st>>>(len32, len64, n_tu);
    OCB_TRY("pp: out scan",
            cub::DeviceScan::ExclusiveSum(ctx->cub_tmp.p, t2, len64, d_out_off, (int)n1, st));
    uint64_t total = 0;
    OCB_TRY("pp: d2h", cudaMemcpyAsync(&total, d_out_off + n_tu, 8, cudaMemcpyDeviceToHost, st));
    OCB_TRY("pp: sync", stream_wait(st));
    OCB_TRY("pp: output", out_text.ensure(total + 64));
    k_pp_pack<<<n_tu, 128, 0, st>>>(ctx->pp_arena.as<uint8_t>(), arena_off, d_out_off,
                                    out_text.as<uint8_t>(), n_tu);
    OCB_TRY("pp: launch", cudaGetLastError());
    *h_total = total;
    return 0;
}

}  // namespace ocb
