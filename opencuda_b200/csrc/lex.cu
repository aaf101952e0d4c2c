// Batch lexer for sm_100a: host driver (kernels in lex_kernels.cuh).
#include <cub/cub.cuh>
#include <thrust/iterator/reverse_iterator.h>
#include "ocb_internal.h"
#include "lex_kernels.cuh"

namespace ocb {

int lex_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t N, const uint64_t *d_tu_off,
               uint32_t n_tu, uint32_t *d_start, uint32_t *d_kindlen, uint32_t *d_line,
               uint64_t tok_cap, uint64_t *d_tu_tok_off, int32_t *d_status, uint64_t *d_n_tok,
               cudaStream_t st) {
    using namespace lex;
    if (n_tu == 0) {
        OCB_TRY("lex: zero TUs", cudaMemsetAsync(d_n_tok, 0, 8, st));
        OCB_TRY("lex: zero TUs", cudaMemsetAsync(d_tu_tok_off, 0, 8, st));
        return 0;
    }
    if (((uintptr_t)d_src & 15) != 0) return fail(ctx, "lex: source buffer must be 16-byte aligned");
    if (N >= (1ull << 32)) return fail(ctx, "lex: batch larger than 4 GiB");
    if (!ctx->kw_ready) {
        KwEntry t[128];
        build_kw_table(t);
        OCB_TRY("lex: keyword table", cudaMemcpyToSymbol(g_kw, t, sizeof(t)));
        ctx->kw_ready = true;
    }
    uint64_t n_win = (N + WIN - 1) / WIN;
    // scratch layout
    uint64_t nw1 = n_win + 1;
    size_t need = sizeof(uint64_t) * (6 * nw1 + 2 * (uint64_t)n_tu + 4) + sizeof(uint32_t) * nw1;
    OCB_TRY("lex: scratch", ctx->lex_scratch.ensure(need));
    uint64_t *maps = ctx->lex_scratch.as<uint64_t>();
    uint64_t *mapscan = maps + nw1;
    uint64_t *nlseg = mapscan + nw1;
    uint64_t *nlcarry = nlseg + nw1;
    uint64_t *S = nlcarry + nw1;      // n_win + 1 sync points
    uint64_t *counts = S + nw1;       // n_win + 1; holds first-sync values before counting
    unsigned long long *errkey = (unsigned long long *)(counts + nw1);
    uint32_t *unsup = (uint32_t *)(errkey + n_tu);
    uint32_t *sinfo = unsup + n_tu;
    uint64_t *toff = mapscan;         // mapscan is dead once sync info is built
    uint64_t *total = toff + n_win;
    uint64_t *fsync = counts;

    LexOut o{d_start, d_kindlen, d_line, tok_cap, d_tu_tok_off, errkey, unsup};
    unsigned grid_tu = (n_tu + 255) / 256;
    k_fill_u64<<<grid_tu, 256, 0, st>>>((uint64_t *)errkey, n_tu, ~0ull);
    OCB_TRY("lex: memset", cudaMemsetAsync(unsup, 0, sizeof(uint32_t) * n_tu, st));

    if (N == 0) {
        k_lex_all_empty<<<grid_tu, 256, 0, st>>>(n_tu, o);
        k_lex_finish<<<grid_tu, 256, 0, st>>>(n_tu, errkey, unsup, d_status, d_tu_tok_off,
                                               nullptr, d_n_tok);
        OCB_TRY("lex: launch", cudaGetLastError());
        return 0;
    }
    if (n_win >= (1ull << 31)) return fail(ctx, "lex: batch too large");
    unsigned grid = (unsigned)((n_win + BLOCK - 1) / BLOCK);
    int nwi = (int)n_win;

    // cub scratch: the largest of the four scans
    size_t t1 = 0, t2 = 0, t3 = 0, t4 = 0;
    auto rin = thrust::make_reverse_iterator(fsync + n_win);
    auto rout = thrust::make_reverse_iterator(S + n_win);
    cub::DeviceScan::InclusiveScan(nullptr, t1, maps, mapscan, ComposeOp(), nwi, st);
    cub::DeviceScan::ExclusiveScan(nullptr, t2, nlseg, nlcarry, SegSumOp(), (uint64_t)0, nwi, st);
    cub::DeviceScan::InclusiveScan(nullptr, t3, rin, rout, MinOp(), nwi, st);
    cub::DeviceScan::ExclusiveSum(nullptr, t4, counts, toff, nwi + 1, st);
    size_t tmax = t1 > t2 ? t1 : t2;
    tmax = tmax > t3 ? tmax : t3;
    tmax = tmax > t4 ? tmax : t4;
    OCB_TRY("lex: cub scratch", ctx->cub_tmp.ensure(tmax));
    void *tmp = ctx->cub_tmp.p;

    k_lex_map<<<grid, BLOCK, 0, st>>>(d_src, N, d_tu_off, n_tu, n_win, maps);
    OCB_TRY("lex: map scan", cub::DeviceScan::InclusiveScan(tmp, t1, maps, mapscan, ComposeOp(), nwi, st));
    k_lex_sync<<<grid, BLOCK, 0, st>>>(d_src, N, d_tu_off, n_tu, n_win, mapscan, nlseg, fsync, sinfo);
    OCB_TRY("lex: line scan",
            cub::DeviceScan::ExclusiveScan(tmp, t2, nlseg, nlcarry, SegSumOp(), (uint64_t)0, nwi, st));
    OCB_TRY("lex: sync scan", cub::DeviceScan::InclusiveScan(tmp, t3, rin, rout, MinOp(), nwi, st));
    k_set_u64<<<1, 1, 0, st>>>(S + n_win, N);
    k_lex_tokens<<<grid, BLOCK, 0, st>>>(false, d_src, N, d_tu_off, n_tu, n_win, S, sinfo, nlcarry,
                                         counts, nullptr, o);
    k_set_u64<<<1, 1, 0, st>>>(counts + n_win, 0);
    OCB_TRY("lex: count scan", cub::DeviceScan::ExclusiveSum(tmp, t4, counts, toff, nwi + 1, st));
    k_lex_tokens<<<grid, BLOCK, 0, st>>>(true, d_src, N, d_tu_off, n_tu, n_win, S, sinfo, nlcarry,
                                         nullptr, toff, o);
    k_lex_finish<<<grid_tu, 256, 0, st>>>(n_tu, errkey, unsup, d_status, d_tu_tok_off, total,
                                           d_n_tok);
    OCB_TRY("lex: launch", cudaGetLastError());
    return 0;
}

}  // namespace ocb
