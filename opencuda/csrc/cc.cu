// Batch compiler back half for sm_100a, host driver: lex the preprocessed
// text, then parse -> optimize -> emit (the three kernels of cc_k_*.cu) one
// thread per translation unit.  Each TU gets a private slice of one arena
// buffer sized from its token count; a TU that outgrows it reports
// OCB_TU_OVERFLOW and the caller runs it again with a larger slice.
#include <algorithm>
#include <cub/cub.cuh>
#include "ocb_internal.h"
#include "cc_state.cuh"

namespace ocb {
namespace cc {

cudaError_t launch_k_cc_parse(const CCArgs &A, unsigned grid, unsigned block, cudaStream_t st);
cudaError_t launch_k_cc_opt(const CCArgs &A, unsigned grid, unsigned block, cudaStream_t st);
cudaError_t launch_k_cc_emit(const CCArgs &A, unsigned grid, unsigned block, cudaStream_t st);
cudaError_t launch_k_cc_verify(const CCArgs &A, int check_reach, unsigned grid, unsigned block,
                               cudaStream_t st);
const void *k_cc_parse_entry();
const void *k_cc_opt_entry();
const void *k_cc_emit_entry();

// The compiler kernels use no shared memory and wait mostly on loads of their
// TU's IR, so the unified L1/shared array is offered to L1 (carveout 0 = all
// of it).  OCB_CC_CARVEOUT selects another percentage, -1 leaves the driver's
// choice.  Set once per process.
static cudaError_t cc_set_carveout() {
    static int done = 0;
    if (done) return cudaSuccess;
    const char *v = getenv("OCB_CC_CARVEOUT");
    long c = (v && *v) ? atol(v) : 0;
    if (c >= 0) {
        if (c > 100) c = 100;
        const void *fs[3] = {k_cc_parse_entry(), k_cc_opt_entry(), k_cc_emit_entry()};
        for (const void *f : fs) {
            cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, (int)c);
            if (e != cudaSuccess) return e;
        }
    }
    done = 1;
    return cudaSuccess;
}

// Stages beyond CC_STAGE_PTX: the IR verifier's error text after parse (3)
// or after optimize (4); 5 and 6 are the same with check_reachability.
enum { CC_STAGE_VERIFY_IR = 3, CC_STAGE_VERIFY_OPT = 4, CC_STAGE_VERIFY_IR_REACH = 5,
       CC_STAGE_VERIFY_OPT_REACH = 6 };
inline bool stage_runs_opt(int stage) {
    return stage == CC_STAGE_OPT || stage == CC_STAGE_PTX || stage == CC_STAGE_VERIFY_OPT ||
           stage == CC_STAGE_VERIFY_OPT_REACH;
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

// The batch gathered into processing order: TU perm[j] to position j; one
// block per TU.
__global__ void k_cc_gather(const uint8_t *src, const uint64_t *off, const uint32_t *perm,
                            const uint64_t *poff, uint8_t *dst, uint32_t n_tu) {
    uint32_t j = blockIdx.x;
    if (j >= n_tu) return;
    const uint8_t *s = src + off[perm[j]];
    uint8_t *d = dst + poff[j];
    uint64_t n = poff[j + 1] - poff[j];
    for (uint64_t k = threadIdx.x; k < n; k += blockDim.x) d[k] = s[k];
}

// st_p[j] = st[perm[j]]: the earlier stages' verdicts in processing order
__global__ void k_cc_permute_status(const uint32_t *perm, const int32_t *st, int32_t *st_p,
                                    uint32_t n) {
    uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n) st_p[j] = st[perm[j]];
}

// Back to input order: verdicts, output lengths and output slice offsets of
// position j belong to TU perm[j]; len[n] = 0 closes the length scan.
__global__ void k_cc_unpermute(const uint32_t *perm, const int32_t *st_p, const uint64_t *len_p,
                               const uint64_t *cap_p, int32_t *st, uint64_t *len, uint64_t *cap,
                               uint32_t n) {
    uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n) {
        uint32_t i = perm[j];
        st[i] = st_p[j];
        len[i] = len_p[j];
        cap[i] = cap_p[j];
    } else if (j == n) {
        len[n] = 0;
    }
}

}  // namespace cc

// Device stack for the recursive-descent parser: frames are bounded by
// cc::MAX_NEST (expression and statement nesting).
static constexpr size_t kCCStack = 64 * 1024;

static uint64_t env_u64(const char *name, uint64_t dflt) {
    const char *v = getenv(name);
    if (!v || !*v) return dflt;
    return strtoull(v, nullptr, 10);
}

// Compile a batch: gather its TUs largest first, lex them, then
// parse/optimize/emit in chunks of consecutive TUs whose per-TU arena slices
// (sized from the token count) fit a memory budget.  The chunks run on
// several streams, each with its own arena, so the longest compiles (the
// first chunks) overlap with the rest of the batch instead of forming a tail
// of every chunk.  Every TU writes into its own slice of one output buffer;
// at the end the texts are packed back to back in input order into
// `out_text` with d_out_off[n_tu+1], and the verdicts go to d_status in input
// order.
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
    PhaseTimer T(st);
    // processing order: largest source first (stable), OCB_CC_ORDER=0 keeps input order
    std::vector<uint64_t> h_off(n1);
    OCB_TRY("cc: d2h", cudaMemcpyAsync(h_off.data(), d_off, 8 * n1, cudaMemcpyDeviceToHost, st));
    OCB_TRY("cc: sync", stream_wait(st));
    std::vector<uint32_t> h_perm(n_tu);
    for (uint32_t i = 0; i < n_tu; ++i) h_perm[i] = i;
    if (env_u64("OCB_CC_ORDER", 1) != 0)
        std::stable_sort(h_perm.begin(), h_perm.end(), [&](uint32_t x, uint32_t y) {
            return h_off[x + 1] - h_off[x] > h_off[y + 1] - h_off[y];
        });
    std::vector<uint64_t> h_poff(n1);
    h_poff[0] = 0;
    for (uint32_t j = 0; j < n_tu; ++j)
        h_poff[j + 1] = h_poff[j] + (h_off[h_perm[j] + 1] - h_off[h_perm[j]]);
    // meta: perm u32[n1] | poff | len_p | cap_p | len_o | cap_o (u64[n1] each)
    //       | st_p i32[n1] | arena offsets u64[2 n1]
    size_t m_perm = (4 * n1 + 15) & ~(size_t)15;
    size_t m_u64 = 8 * n1;
    size_t m_st = (4 * n1 + 15) & ~(size_t)15;
    OCB_TRY("cc: meta", ctx->cc_pmeta.ensure(m_perm + 5 * m_u64 + m_st + 16 * n1 + 64));
    uint8_t *mb = ctx->cc_pmeta.as<uint8_t>();
    uint32_t *perm = (uint32_t *)mb;
    uint64_t *poff = (uint64_t *)(mb + m_perm);
    uint64_t *len_p = poff + n1;
    uint64_t *cap_p = len_p + n1;
    uint64_t *len_o = cap_p + n1;
    uint64_t *cap_o = len_o + n1;
    int32_t *st_p = (int32_t *)(cap_o + n1);
    uint64_t *aoff_all = (uint64_t *)((uint8_t *)st_p + m_st);
    OCB_TRY("cc: text", ctx->cc_ptext.ensure(N + 64));
    uint8_t *ptext = ctx->cc_ptext.as<uint8_t>();
    OCB_TRY("cc: h2d", cudaMemcpyAsync(perm, h_perm.data(), 4 * (size_t)n_tu,
                                       cudaMemcpyHostToDevice, st));
    OCB_TRY("cc: h2d", cudaMemcpyAsync(poff, h_poff.data(), 8 * n1, cudaMemcpyHostToDevice, st));
    k_cc_gather<<<n_tu, 256, 0, st>>>(d_text, d_off, perm, poff, ptext, n_tu);
    OCB_TRY("cc: gather", cudaGetLastError());
    // lex the gathered batch (token starts are offsets into ptext)
    uint64_t tok_cap = N + n_tu + 16;
    OCB_TRY("cc: tokens", ctx->cc_tok.ensure(12 * tok_cap + 16));
    OCB_TRY("cc: scratch", ctx->cc_scratch.ensure(8 * n1 + 8 + 4 * n1 + 64 +
                                                  16 * ocb_ctx::kCCStreams + 16));
    uint32_t *tstart = ctx->cc_tok.as<uint32_t>();
    uint32_t *tkl = tstart + tok_cap;
    uint64_t *tu_tok = ctx->cc_scratch.as<uint64_t>();
    uint64_t *n_tok = tu_tok + n1;
    int32_t *lex_status = (int32_t *)(n_tok + 1);
    unsigned long long *spill_top =
        (unsigned long long *)(((uintptr_t)(lex_status + n1) + 15) & ~(uintptr_t)15);
    int rc = lex_device(ctx, ptext, N, poff, n_tu, tstart, tkl, nullptr, tok_cap, tu_tok,
                        lex_status, n_tok, st);
    if (rc) return rc;
    T.mark("cc: lex");
    unsigned grid = (unsigned)((n1 + 255) / 256);
    k_cc_permute_status<<<grid, 256, 0, st>>>(perm, d_in_status, st_p, n_tu);
    merge_status<<<grid, 256, 0, st>>>(st_p, lex_status, n_tu);
    OCB_TRY("cc: status", cudaGetLastError());
    std::vector<uint64_t> h_tok(n1);
    OCB_TRY("cc: d2h", cudaMemcpyAsync(h_tok.data(), tu_tok, 8 * n1, cudaMemcpyDeviceToHost, st));
    OCB_TRY("cc: sync", stream_wait(st));
    OCB_TRY("cc: carveout", cc_set_carveout());
    size_t cur_stack = 0;
    OCB_TRY("cc: stack limit", cudaDeviceGetLimit(&cur_stack, cudaLimitStackSize));
    if (cur_stack < kCCStack) OCB_TRY("cc: stack limit", cudaDeviceSetLimit(cudaLimitStackSize, kCCStack));
    // sizing (bytes per token of the TU, times the retry scale)
    // Measured on generated kernels: the IR peaks near 500-750 B/token and the
    // optimizer's per-pass scratch near 650-1300 B/token (p50-p99); PTX text is
    // 11-16 B/token.  A TU beyond these reruns with every size times 8.
    uint64_t a0 = env_u64("OCB_CC_ARENA_BASE", 32768), a1 = env_u64("OCB_CC_ARENA_PER_TOKEN", 2400);
    uint64_t o0 = 4096, o1 = env_u64("OCB_CC_OUT_PER_TOKEN", stage == CC_STAGE_PTX ? 40 : 200);
    uint32_t ir_pm = (uint32_t)env_u64("OCB_CC_IR_PERMILLE", 400);
    uint32_t spread = (uint32_t)env_u64("OCB_CC_SPREAD", 1);
    if (spread < 1) spread = 1;
    if (spread > 32) spread = 32;
    // Threads per block of the compiler kernels (one TU per warp): 128 by
    // default.  One warp per block (32) frees a TU's registers the moment it
    // finishes and spreads a chunk's largest TUs over SMs, but measured 2%
    // slower on the lognormal batch (20.1 against 20.6 MB/s, same box).
    unsigned bthreads = (unsigned)env_u64("OCB_CC_BLOCK", 128);
    if (bthreads != 32 && bthreads != 64) bthreads = 128;
    // every TU's output slice, in processing order, in one buffer
    std::vector<uint64_t> h_cap(n1);
    h_cap[0] = 0;
    for (uint32_t j = 0; j < n_tu; ++j)
        h_cap[j + 1] = h_cap[j] + (((o0 + o1 * (h_tok[j + 1] - h_tok[j])) * scale + 15) & ~15ull);
    size_t free_b = 0, total_b = 0;
    OCB_TRY("cc: meminfo", cudaMemGetInfo(&free_b, &total_b));
    uint64_t owned = ctx->cc_out.cap;
    for (int q = 0; q < ocb_ctx::kCCStreams; ++q) owned += ctx->cc_arena_s[q].cap + ctx->cc_spill_s[q].cap;
    uint64_t budget = (uint64_t)((double)(free_b + owned) * 0.45);
    uint64_t budget_cap = env_u64("OCB_CC_BUDGET_MB", 73728) << 20;
    if (budget > budget_cap) budget = budget_cap;
    uint64_t out_total = h_cap[n_tu] + 64;
    OCB_TRY("cc: out", ctx->cc_out.ensure(out_total));
    uint64_t arena_budget = budget > out_total + (768ull << 20) ? budget - out_total : (768ull << 20);
    int S = (int)env_u64("OCB_CC_STREAMS", 3);
    if (S < 1) S = 1;
    if (S > ocb_ctx::kCCStreams) S = ocb_ctx::kCCStreams;
    uint64_t per_stream = arena_budget / S;
    if (per_stream < (256ull << 20)) per_stream = 256ull << 20;
    // One eighth of a stream's budget is the spill pool that its TUs outgrowing
    // their slice draw from (shared by every TU of a chunk, reset per chunk).
    uint64_t spill_b = env_u64("OCB_CC_SPILL_MB", per_stream >> 23) << 20;
    uint64_t slice_budget = per_stream - (spill_b < per_stream / 2 ? spill_b : per_stream / 2);
    // chunks: consecutive TUs of the processing order whose slices fit
    std::vector<uint32_t> ch_a;
    std::vector<uint64_t> h_aoff_all;
    h_aoff_all.reserve(2 * n1);
    uint64_t stream_need[ocb_ctx::kCCStreams] = {};
    for (uint32_t a = 0; a < n_tu;) {
        ch_a.push_back(a);
        uint64_t run = 0;
        h_aoff_all.push_back(0);
        uint32_t b = a;
        while (b < n_tu) {
            uint64_t as = ((a0 + a1 * (h_tok[b + 1] - h_tok[b])) * scale + 15) & ~15ull;
            if (b > a && run + as > slice_budget) break;
            run += as;
            h_aoff_all.push_back(run);
            ++b;
        }
        int s_ = (int)((ch_a.size() - 1) % S);
        if (run + 64 > stream_need[s_]) stream_need[s_] = run + 64;
        a = b;
    }
    ch_a.push_back(n_tu);
    size_t n_ch = ch_a.size() - 1;
    OCB_TRY("cc: h2d", cudaMemcpyAsync(cap_p, h_cap.data(), 8 * n1, cudaMemcpyHostToDevice, st));
    OCB_TRY("cc: h2d", cudaMemcpyAsync(aoff_all, h_aoff_all.data(), 8 * h_aoff_all.size(),
                                       cudaMemcpyHostToDevice, st));
    OCB_TRY("cc: zero", cudaMemsetAsync(len_p, 0, 8 * n1, st));
    OCB_TRY("cc: zero", cudaMemsetAsync(spill_top, 0, 16 * ocb_ctx::kCCStreams, st));
    int used_streams = n_ch < (size_t)S ? (int)n_ch : S;
    for (int q = 0; q < used_streams; ++q) {
        if (!ctx->cc_streams[q])
            OCB_TRY("cc: stream", cudaStreamCreateWithFlags(&ctx->cc_streams[q], cudaStreamNonBlocking));
        OCB_TRY("cc: arena", ctx->cc_arena_s[q].ensure(stream_need[q]));
        if (spill_b) OCB_TRY("cc: spill pool", ctx->cc_spill_s[q].ensure(spill_b));
    }
    cudaEvent_t ready;
    OCB_TRY("cc: event", cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
    OCB_TRY("cc: event", cudaEventRecord(ready, st));
    for (int q = 0; q < used_streams; ++q)
        OCB_TRY("cc: event", cudaStreamWaitEvent(ctx->cc_streams[q], ready, 0));
    T.mark("cc: setup");
    bool kp = ctx->kprof_on;
    std::vector<cudaEvent_t> kev;
    if (kp) {
        kev.resize(4 * n_ch);
        for (auto &e : kev) OCB_TRY("cc: event", cudaEventCreate(&e));
    }
    unsigned long long *tops = spill_top;
    for (size_t c = 0; c < n_ch; ++c) {
        int q = (int)(c % S);
        cudaStream_t ss = ctx->cc_streams[q];
        uint32_t a = ch_a[c], nc = ch_a[c + 1] - a;
        if (c >= (size_t)S)  // the stream's previous chunk drew on the same spill pool
            OCB_TRY("cc: zero", cudaMemsetAsync(tops + 2 * q, 0, 8, ss));
        CCArgs A{ptext, tstart, tkl, tu_tok + a, nc, ctx->cc_arena_s[q].as<uint8_t>(),
                 aoff_all + a + c, ctx->cc_out.as<uint8_t>(), cap_p + a, len_p + a, st_p + a,
                 stage, spread, ir_pm, nullptr, {}, nullptr,
                 SpillPool{spill_b ? ctx->cc_spill_s[q].as<uint8_t>() : nullptr,
                           spill_b ? tops + 2 * q : nullptr, spill_b}};
        memcpy(A.target, ctx->target, sizeof A.target);
        unsigned warps = (nc + spread - 1) / spread;
        unsigned blocks = (warps * 32 + bthreads - 1) / bthreads;
        if (kp) OCB_TRY("cc: event", cudaEventRecord(kev[4 * c], ss));
        OCB_TRY("cc: parse launch", launch_k_cc_parse(A, blocks, bthreads, ss));
        if (kp) OCB_TRY("cc: event", cudaEventRecord(kev[4 * c + 1], ss));
        if (stage_runs_opt(stage)) OCB_TRY("cc: optimize launch", launch_k_cc_opt(A, blocks, bthreads, ss));
        if (kp) OCB_TRY("cc: event", cudaEventRecord(kev[4 * c + 2], ss));
        if (stage <= CC_STAGE_PTX)
            OCB_TRY("cc: emit launch", launch_k_cc_emit(A, blocks, bthreads, ss));
        else
            OCB_TRY("cc: verify launch",
                    launch_k_cc_verify(A, stage >= CC_STAGE_VERIFY_IR_REACH, blocks, bthreads, ss));
        if (kp) OCB_TRY("cc: event", cudaEventRecord(kev[4 * c + 3], ss));
    }
    for (int q = 0; q < used_streams; ++q) {
        OCB_TRY("cc: event", cudaEventRecord(ready, ctx->cc_streams[q]));
        OCB_TRY("cc: event", cudaStreamWaitEvent(st, ready, 0));
    }
    cudaEventDestroy(ready);
    T.mark("cc: chunks");
    // back to input order, then the texts packed back to back
    k_cc_unpermute<<<grid, 256, 0, st>>>(perm, st_p, len_p, cap_p, d_status, len_o, cap_o, n_tu);
    OCB_TRY("cc: unpermute", cudaGetLastError());
    size_t t1 = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, t1, len_o, d_out_off, (int)n1, st);
    OCB_TRY("cc: cub scratch", ctx->cub_tmp.ensure(t1));
    OCB_TRY("cc: pack scan",
            cub::DeviceScan::ExclusiveSum(ctx->cub_tmp.p, t1, len_o, d_out_off, (int)n1, st));
    uint64_t tot = 0;
    OCB_TRY("cc: d2h", cudaMemcpyAsync(&tot, d_out_off + n_tu, 8, cudaMemcpyDeviceToHost, st));
    OCB_TRY("cc: sync", stream_wait(st));
    if (kp) {
        for (size_t c = 0; c < n_ch; ++c)
            for (int k = 0; k < 3; ++k) {
                if (k == 1 && !stage_runs_opt(stage)) continue;
                float ms = 0;
                OCB_TRY("cc: event time", cudaEventElapsedTime(&ms, kev[4 * c + k], kev[4 * c + k + 1]));
                ctx->kms[k] += ms;
                ctx->kn[k] += 1;
            }
        for (auto &e : kev) cudaEventDestroy(e);
    }
    OCB_TRY("cc: output", out_text.ensure(tot + 64));
    cc::k_cc_pack<<<n_tu, 128, 0, st>>>(ctx->cc_out.as<uint8_t>(), cap_o, d_out_off,
                                        out_text.as<uint8_t>(), n_tu);
    OCB_TRY("cc: pack launch", cudaGetLastError());
    OCB_TRY("cc: sync", stream_wait(st));
    T.mark("cc: pack");
    *h_total = tot;
    return 0;
}
}  // namespace ocb
