// Batch lexer for sm_100a: host driver (kernels in lex_kernels.cuh).
#include <cstdlib>
#include <cub/cub.cuh>
#include <thrust/iterator/reverse_iterator.h>
#include "ocb_internal.h"
#include "lex_kernels.cuh"
#include "lex_fused.cuh"

namespace ocb {

// The single-pass lexer (lex_fused.cuh): token records without lines.
static int lex_device_fused(ocb_ctx *ctx, const uint8_t *d_src, uint64_t N,
                            const uint64_t *d_tu_off, uint32_t n_tu, uint32_t *d_start,
                            uint32_t *d_kindlen, uint64_t tok_cap, uint64_t *d_tu_tok_off,
                            int32_t *d_status, uint64_t *d_n_tok, cudaStream_t st) {
    using namespace lex;
    uint64_t n_win = (N + WIN - 1) / WIN;
    uint64_t n_tiles = (n_win + FT - 1) / FT;
    // scratch: errkey[n_tu] | unsup[n_tu] | ticket, err | mstat[n_tiles] | cstat[n_tiles]
    size_t a_err = (8 * (size_t)n_tu + 4 * (size_t)n_tu + 15) & ~(size_t)15;
    size_t zero_bytes = 16 + 16 * (size_t)n_tiles;
    OCB_TRY("lex: scratch", ctx->lex_scratch.ensure(a_err + zero_bytes));
    uint8_t *base = ctx->lex_scratch.as<uint8_t>();
    unsigned long long *errkey = (unsigned long long *)base;
    uint32_t *unsup = (uint32_t *)(errkey + n_tu);
    unsigned long long *ticket = (unsigned long long *)(base + a_err);
    unsigned int *err = (unsigned int *)(ticket + 1);
    unsigned long long *mstat = ticket + 2;
    unsigned long long *cstat = mstat + n_tiles;
    unsigned grid_tu = (n_tu + 255) / 256;
    k_fill_u64<<<grid_tu, 256, 0, st>>>((uint64_t *)errkey, n_tu, ~0ull);
    OCB_TRY("lex: memset", cudaMemsetAsync(unsup, 0, sizeof(uint32_t) * n_tu, st));
    OCB_TRY("lex: memset", cudaMemsetAsync(ticket, 0, zero_bytes, st));
    int dev = 0, n_sm = 0, per_sm = 0;
    OCB_TRY("lex: device", cudaGetDevice(&dev));
    OCB_TRY("lex: device", cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev));
    OCB_TRY("lex: occupancy",
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_lex_fused, FT, 0));
    if (per_sm < 1) per_sm = 1;
    uint64_t grid = (uint64_t)n_sm * per_sm;
    if (grid > n_tiles) grid = n_tiles;
    LexOut o{d_start, d_kindlen, nullptr, tok_cap, d_tu_tok_off, errkey, unsup};
    FusedArgs A{d_src, N, d_tu_off, n_tu, n_win, n_tiles, ticket, mstat, cstat, err, o, d_n_tok};
    k_lex_fused<<<(unsigned)grid, FT, 0, st>>>(A);
    k_lex_fused_finish<<<grid_tu, 256, 0, st>>>(n_tu, errkey, unsup, err, d_status);
    OCB_TRY("lex: launch", cudaGetLastError());
    return 0;
}

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
    // Without per-token lines the single-pass kernel does the whole job
    // (OCB_LEX_FUSED=0 selects the multi-pass pipeline, for comparisons).
    const char *fv = getenv("OCB_LEX_FUSED");
    if (!d_line && N > 0 && !(fv && *fv == '0'))
        return lex_device_fused(ctx, d_src, N, d_tu_off, n_tu, d_start, d_kindlen, tok_cap,
                                d_tu_tok_off, d_status, d_n_tok, st);
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
    // OCB_LEX_MATCHER=1 selects the sequential matcher (for timing comparisons)
    const char *mv = getenv("OCB_LEX_MATCHER");
    bool dfa = !(mv && *mv && *mv != '0');
    if (dfa)
        k_lex_tokens_dfa<<<grid, BLOCK, 0, st>>>(false, d_src, N, d_tu_off, n_tu, n_win, S, sinfo,
                                                 nlcarry, counts, nullptr, o);
    else
        k_lex_tokens<<<grid, BLOCK, 0, st>>>(false, d_src, N, d_tu_off, n_tu, n_win, S, sinfo,
                                             nlcarry, counts, nullptr, o);
    k_set_u64<<<1, 1, 0, st>>>(counts + n_win, 0);
    OCB_TRY("lex: count scan", cub::DeviceScan::ExclusiveSum(tmp, t4, counts, toff, nwi + 1, st));
    if (dfa)
        k_lex_tokens_dfa<<<grid, BLOCK, 0, st>>>(true, d_src, N, d_tu_off, n_tu, n_win, S, sinfo,
                                                 nlcarry, nullptr, toff, o);
    else
        k_lex_tokens<<<grid, BLOCK, 0, st>>>(true, d_src, N, d_tu_off, n_tu, n_win, S, sinfo,
                                             nlcarry, nullptr, toff, o);
    k_lex_finish<<<grid_tu, 256, 0, st>>>(n_tu, errkey, unsup, d_status, d_tu_tok_off, total,
                                           d_n_tok);
    OCB_TRY("lex: launch", cudaGetLastError());
    return 0;
}

}  // namespace ocb

// ---------------------------------------------------------------------------
// Allocation-free lexer entry point.
//
// Some callers cannot allocate device memory at the moment they lex: code
// running inside another framework's memory pool or a pre-sized arena that
// forbids cudaMalloc/cudaFree after start-up, or a host thread that must not
// take the allocator's global lock.  For them the whole lexer pipeline runs
// with its scratch in one fixed device array compiled into this library; the
// caller passes only inputs and outputs.
// ---------------------------------------------------------------------------
#include <cstring>
#include <mutex>

namespace ocb {
namespace {

constexpr uint64_t kStaticMaxBytes = 4ull << 20;   // source bytes per call
constexpr uint32_t kStaticMaxTus = 16384;          // TUs per call
constexpr size_t kStaticScratchBytes = 8ull << 20; // size of the array below

// Held by every GPU that loads the library, until the process exits.  Host
// code must not pass this name to a kernel (on the host it is only a stand-in
// symbol); the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_lex_static_scratch[kStaticScratchBytes];

// The fixed part of the layout (per-window and per-TU arrays) at the limits
// must leave room for the scan scratch that follows it.
constexpr size_t kStaticFixedMax =
    ((sizeof(uint64_t) * (6 * (kStaticMaxBytes / lex::WIN + 2) + 2 * (uint64_t)kStaticMaxTus + 4) +
      sizeof(uint32_t) * (kStaticMaxBytes / lex::WIN + 2)) + 255) & ~(size_t)255;
static_assert(kStaticFixedMax + (1u << 20) <= kStaticScratchBytes,
              "static lexer scratch: the fixed layout at the limits leaves under 1 MiB for scans");

constexpr int kMaxDevices = 128;
std::mutex g_static_mu;
void *g_static_ptr[kMaxDevices];  // device address of the array, per device

int static_fail(char *err, size_t err_len, int code, const char *msg) {
    if (err && err_len) {
        strncpy(err, msg, err_len - 1);
        err[err_len - 1] = 0;
    }
    return code;
}

}  // namespace
}  // namespace ocb

extern "C" int ocb_lex_device_static(const uint8_t *d_src, uint64_t N, const uint64_t *d_tu_off,
                                     uint32_t n_tu, uint32_t *d_start, uint32_t *d_kindlen,
                                     uint32_t *d_line, uint64_t tok_cap, uint64_t *d_tu_tok_off,
                                     int32_t *d_status, uint64_t *d_n_tok, void *stream,
                                     char *err, size_t err_len) {
    using namespace ocb;
    using namespace ocb::lex;
    cudaStream_t st = (cudaStream_t)stream;
    if (err && err_len) err[0] = 0;
    if (N > kStaticMaxBytes)
        return static_fail(err, err_len, -2,
                           "ocb_lex_device_static: batch exceeds 4 MiB of source "
                           "(use ocb_lex_device for larger batches)");
    if (n_tu > kStaticMaxTus)
        return static_fail(err, err_len, -2,
                           "ocb_lex_device_static: batch exceeds 16384 TUs "
                           "(use ocb_lex_device for larger batches)");
    if (((uintptr_t)d_src & 15) != 0)
        return static_fail(err, err_len, -1, "ocb_lex_device_static: source must be 16-byte aligned");
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return static_fail(err, err_len, -1, "ocb_lex_device_static: no current CUDA device");
    void *base = nullptr;
    {
        // Set-up on this device (the current one): the array's device address
        // and the keyword table.  Neither allocates.  The address is looked up
        // on every call: after a device reset (a new primary context) it can
        // change and the keyword table is gone, so a changed address redoes
        // the upload.
        std::lock_guard<std::mutex> lock(g_static_mu);
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_lex_static_scratch) != cudaSuccess || !p)
            return static_fail(err, err_len, -1,
                               "ocb_lex_device_static: cudaGetSymbolAddress failed");
        if (g_static_ptr[dev] != p) {
            KwEntry t[128];
            build_kw_table(t);
            if (cudaMemcpyToSymbol(g_kw, t, sizeof(t)) != cudaSuccess)
                return static_fail(err, err_len, -1,
                                   "ocb_lex_device_static: keyword table upload failed");
            g_static_ptr[dev] = p;
        }
        base = g_static_ptr[dev];
    }
    if (n_tu == 0) {
        if (cudaMemsetAsync(d_n_tok, 0, 8, st) != cudaSuccess ||
            cudaMemsetAsync(d_tu_tok_off, 0, 8, st) != cudaSuccess)
            return static_fail(err, err_len, -1, "ocb_lex_device_static: memset failed");
        return 0;
    }
    uint64_t n_win = (N + WIN - 1) / WIN, nw1 = n_win + 1;
    size_t fixed = sizeof(uint64_t) * (6 * nw1 + 2 * (uint64_t)n_tu + 4) + sizeof(uint32_t) * nw1;
    fixed = (fixed + 255) & ~(size_t)255;
    uint64_t *maps = (uint64_t *)base;
    uint64_t *mapscan = maps + nw1;
    uint64_t *nlseg = mapscan + nw1;
    uint64_t *nlcarry = nlseg + nw1;
    uint64_t *S = nlcarry + nw1;
    uint64_t *counts = S + nw1;
    unsigned long long *errkey = (unsigned long long *)(counts + nw1);
    uint32_t *unsup = (uint32_t *)(errkey + n_tu);
    uint32_t *sinfo = unsup + n_tu;
    uint64_t *toff = mapscan;
    uint64_t *total = toff + n_win;
    uint64_t *fsync = counts;
    if (fixed > kStaticScratchBytes)
        return static_fail(err, err_len, -2, "ocb_lex_device_static: layout exceeds the array");
    void *tmp = (unsigned char *)base + fixed;
    size_t tmp_cap = kStaticScratchBytes - fixed;

    LexOut o{d_start, d_kindlen, d_line, tok_cap, d_tu_tok_off, errkey, unsup};
    unsigned grid_tu = (n_tu + 255) / 256;
    // errkey must start at all-ones and unsup at zero on every call: the array
    // keeps whatever the previous call left in it.
    k_fill_u64<<<grid_tu, 256, 0, st>>>((uint64_t *)errkey, n_tu, ~0ull);
    if (cudaMemsetAsync(unsup, 0, sizeof(uint32_t) * n_tu, st) != cudaSuccess)
        return static_fail(err, err_len, -1, "ocb_lex_device_static: memset failed");
    if (N == 0) {
        k_lex_all_empty<<<grid_tu, 256, 0, st>>>(n_tu, o);
        k_lex_finish<<<grid_tu, 256, 0, st>>>(n_tu, errkey, unsup, d_status, d_tu_tok_off,
                                               nullptr, d_n_tok);
        return cudaGetLastError() == cudaSuccess
                   ? 0 : static_fail(err, err_len, -1, "ocb_lex_device_static: launch failed");
    }
    unsigned grid = (unsigned)((n_win + BLOCK - 1) / BLOCK);
    int nwi = (int)n_win;
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
    if (tmax > tmp_cap)
        return static_fail(err, err_len, -2, "ocb_lex_device_static: scan scratch does not fit");

    // Each step is queued only when everything before it was queued: a
    // failed scan must not leave later kernels reading what an earlier call
    // left in the array and writing it to the caller's outputs.
    const char *failed = "ocb_lex_device_static: launch failed";
    k_lex_map<<<grid, BLOCK, 0, st>>>(d_src, N, d_tu_off, n_tu, n_win, maps);
    if (cudaGetLastError() != cudaSuccess ||
        cub::DeviceScan::InclusiveScan(tmp, t1, maps, mapscan, ComposeOp(), nwi, st) != cudaSuccess)
        return static_fail(err, err_len, -1, failed);
    k_lex_sync<<<grid, BLOCK, 0, st>>>(d_src, N, d_tu_off, n_tu, n_win, mapscan, nlseg, fsync, sinfo);
    if (cudaGetLastError() != cudaSuccess ||
        cub::DeviceScan::ExclusiveScan(tmp, t2, nlseg, nlcarry, SegSumOp(), (uint64_t)0, nwi,
                                       st) != cudaSuccess ||
        cub::DeviceScan::InclusiveScan(tmp, t3, rin, rout, MinOp(), nwi, st) != cudaSuccess)
        return static_fail(err, err_len, -1, failed);
    k_set_u64<<<1, 1, 0, st>>>(S + n_win, N);
    k_lex_tokens_dfa<<<grid, BLOCK, 0, st>>>(false, d_src, N, d_tu_off, n_tu, n_win, S, sinfo,
                                             nlcarry, counts, nullptr, o);
    k_set_u64<<<1, 1, 0, st>>>(counts + n_win, 0);
    if (cudaGetLastError() != cudaSuccess ||
        cub::DeviceScan::ExclusiveSum(tmp, t4, counts, toff, nwi + 1, st) != cudaSuccess)
        return static_fail(err, err_len, -1, failed);
    k_lex_tokens_dfa<<<grid, BLOCK, 0, st>>>(true, d_src, N, d_tu_off, n_tu, n_win, S, sinfo,
                                             nlcarry, nullptr, toff, o);
    k_lex_finish<<<grid_tu, 256, 0, st>>>(n_tu, errkey, unsup, d_status, d_tu_tok_off, total,
                                           d_n_tok);
    if (cudaGetLastError() != cudaSuccess) return static_fail(err, err_len, -1, failed);
    return 0;
}
