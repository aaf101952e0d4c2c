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

// out_off[a + j] = base + pack_off[j] for the chunk's TUs (and the end entry)
__global__ void k_cc_out_off(const uint64_t *pack_off, uint64_t base, uint64_t *out_off, uint32_t n) {
    uint32_t j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j <= n) out_off[j] = base + pack_off[j];
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

// Lex the batch, then parse/optimize/emit it chunk by chunk: each chunk's
// per-TU arena slices (sized from the TU's token count) fit a memory budget
// taken from the free device memory.  Outputs are packed back to back into
// `out_text` with d_out_off[n_tu+1].
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
    OCB_TRY("cc: scratch", ctx->cc_scratch.ensure(8 * n1 * 5 + 8 + 4 * n1 + 64 + 16));
    uint32_t *tstart = ctx->cc_tok.as<uint32_t>();
    uint32_t *tkl = tstart + tok_cap;
    uint32_t *tline = tkl + tok_cap;
    uint64_t *tu_tok = ctx->cc_scratch.as<uint64_t>();
    uint64_t *arena_off = tu_tok + n1;
    uint64_t *out_cap_off = arena_off + n1;
    uint64_t *out_len = out_cap_off + n1;
    uint64_t *pack_off = out_len + n1;
    uint64_t *n_tok = pack_off + n1;
    int32_t *lex_status = (int32_t *)(n_tok + 1);
    unsigned long long *spill_top =
        (unsigned long long *)(((uintptr_t)(lex_status + n1) + 15) & ~(uintptr_t)15);
    PhaseTimer T(st);
    // the parser reads token starts and kinds only: no per-token lines
    (void)tline;
    int rc = lex_device(ctx, d_text, N, d_off, n_tu, tstart, tkl, nullptr, tok_cap, tu_tok,
                        lex_status, n_tok, st);
    if (rc) return rc;
    T.mark("cc: lex");
    OCB_TRY("cc: status", cudaMemcpyAsync(d_status, d_in_status, 4 * (size_t)n_tu,
                                          cudaMemcpyDeviceToDevice, st));
    unsigned grid = (unsigned)((n1 + 255) / 256);
    merge_status<<<grid, 256, 0, st>>>(d_status, lex_status, n_tu);
    std::vector<uint64_t> h_tok(n1);
    OCB_TRY("cc: d2h", cudaMemcpyAsync(h_tok.data(), tu_tok, 8 * n1, cudaMemcpyDeviceToHost, st));
    OCB_TRY("cc: sync", stream_wait(st));
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
    size_t free_b = 0, total_b = 0;
    OCB_TRY("cc: meminfo", cudaMemGetInfo(&free_b, &total_b));
    uint64_t budget = (uint64_t)((double)(free_b + ctx->cc_arena.cap + ctx->cc_out.cap) * 0.45);
    uint64_t budget_cap = env_u64("OCB_CC_BUDGET_MB", 24576) << 20;
    if (budget > budget_cap) budget = budget_cap;
    if (budget < (256ull << 20)) budget = 256ull << 20;
    // One eighth of the budget is the spill pool that TUs outgrowing their
    // slice draw from (shared by every TU of a chunk, reset per chunk).
    uint64_t spill_b = env_u64("OCB_CC_SPILL_MB", budget >> 23) << 20;
    if (spill_b) {
        OCB_TRY("cc: spill pool", ctx->cc_spill.ensure(spill_b));
        budget -= spill_b < budget / 2 ? spill_b : budget / 2;
    }
    bool order_on = env_u64("OCB_CC_ORDER", 1) != 0;
    OCB_TRY("cc: order", ctx->cc_order.ensure(4 * (size_t)n_tu + 16));
    std::vector<uint32_t> h_order;
    std::vector<uint64_t> h_aoff, h_ooff;
    uint64_t running = 0;
    uint32_t a = 0;
    while (a < n_tu) {
        // chunk [a, b): arena + output slices within the budget (at least one TU)
        h_aoff.assign(1, 0);
        h_ooff.assign(1, 0);
        uint32_t b = a;
        while (b < n_tu) {
            uint64_t nt = h_tok[b + 1] - h_tok[b];
            uint64_t as = ((a0 + a1 * nt) * scale + 15) & ~15ull;
            uint64_t os = ((o0 + o1 * nt) * scale + 15) & ~15ull;
            if (b > a && h_aoff.back() + as + h_ooff.back() + os > budget) break;
            h_aoff.push_back(h_aoff.back() + as);
            h_ooff.push_back(h_ooff.back() + os);
            ++b;
        }
        uint32_t nc = b - a;
        OCB_TRY("cc: arena", ctx->cc_arena.ensure(h_aoff.back() + 64));
        OCB_TRY("cc: out", ctx->cc_out.ensure(h_ooff.back() + 64));
        OCB_TRY("cc: h2d", cudaMemcpyAsync(arena_off, h_aoff.data(), 8 * (size_t)(nc + 1),
                                           cudaMemcpyHostToDevice, st));
        OCB_TRY("cc: h2d", cudaMemcpyAsync(out_cap_off, h_ooff.data(), 8 * (size_t)(nc + 1),
                                           cudaMemcpyHostToDevice, st));
        OCB_TRY("cc: zero", cudaMemsetAsync(out_len, 0, 8 * (size_t)(nc + 1), st));
        OCB_TRY("cc: zero", cudaMemsetAsync(spill_top, 0, 8, st));
        if (order_on) {
            // largest TUs (by tokens) first: the longest-running threads start
            // in the first wave instead of forming the tail
            h_order.resize(nc);
            for (uint32_t j = 0; j < nc; ++j) h_order[j] = j;
            std::stable_sort(h_order.begin(), h_order.end(), [&](uint32_t x, uint32_t y) {
                return h_tok[a + x + 1] - h_tok[a + x] > h_tok[a + y + 1] - h_tok[a + y];
            });
            OCB_TRY("cc: h2d", cudaMemcpyAsync(ctx->cc_order.p, h_order.data(), 4 * (size_t)nc,
                                               cudaMemcpyHostToDevice, st));
        }
        CCArgs A{d_text, tstart, tkl, tu_tok + a, nc, ctx->cc_arena.as<uint8_t>(), arena_off,
                 ctx->cc_out.as<uint8_t>(), out_cap_off, out_len, d_status + a, stage, spread,
                 ir_pm, nullptr, {}, order_on ? ctx->cc_order.as<uint32_t>() : nullptr,
                 SpillPool{spill_b ? ctx->cc_spill.as<uint8_t>() : nullptr,
                           spill_b ? spill_top : nullptr, spill_b}};
        memcpy(A.target, ctx->target, sizeof A.target);
        unsigned warps = (nc + spread - 1) / spread;
        unsigned blocks = (warps + 3) / 4;  // 4 warps (128 threads) per block
        T.mark("cc: chunk setup");
        bool kp = ctx->kprof_on;
        if (kp) OCB_TRY("cc: event", cudaEventRecord(ctx->kev[0], st));
        OCB_TRY("cc: parse launch", launch_k_cc_parse(A, blocks, 128, st));
        if (kp) OCB_TRY("cc: event", cudaEventRecord(ctx->kev[1], st));
        T.mark("cc: k_cc_parse");
        if (stage_runs_opt(stage)) OCB_TRY("cc: optimize launch", launch_k_cc_opt(A, blocks, 128, st));
        if (kp) OCB_TRY("cc: event", cudaEventRecord(ctx->kev[2], st));
        T.mark("cc: k_cc_opt");
        if (stage <= CC_STAGE_PTX)
            OCB_TRY("cc: emit launch", launch_k_cc_emit(A, blocks, 128, st));
        else
            OCB_TRY("cc: verify launch",
                    launch_k_cc_verify(A, stage >= CC_STAGE_VERIFY_IR_REACH, blocks, 128, st));
        if (kp) OCB_TRY("cc: event", cudaEventRecord(ctx->kev[3], st));
        T.mark("cc: k_cc_emit");
        size_t t1 = 0;
        cub::DeviceScan::ExclusiveSum(nullptr, t1, out_len, pack_off, (int)(nc + 1), st);
        OCB_TRY("cc: cub scratch", ctx->cub_tmp.ensure(t1));
        OCB_TRY("cc: pack scan",
                cub::DeviceScan::ExclusiveSum(ctx->cub_tmp.p, t1, out_len, pack_off, (int)(nc + 1), st));
        uint64_t tot = 0;
        OCB_TRY("cc: d2h", cudaMemcpyAsync(&tot, pack_off + nc, 8, cudaMemcpyDeviceToHost, st));
        OCB_TRY("cc: sync", stream_wait(st));
        if (kp) {
            for (int k = 0; k < 3; ++k) {
                if (k == 1 && !stage_runs_opt(stage)) continue;
                float ms = 0;
                OCB_TRY("cc: event time", cudaEventElapsedTime(&ms, ctx->kev[k], ctx->kev[k + 1]));
                ctx->kms[k] += ms;
                ctx->kn[k] += 1;
            }
        }
        if (running + tot + 64 > out_text.cap) {  // grow, keeping what is packed so far
            DevBuf nb;
            size_t want = out_text.cap * 2;
            if (want < running + tot + 64) want = running + tot + 64;
            OCB_TRY("cc: output", nb.ensure(want));
            if (running) OCB_TRY("cc: d2d", cudaMemcpyAsync(nb.p, out_text.p, running,
                                                           cudaMemcpyDeviceToDevice, st));
            OCB_TRY("cc: sync", stream_wait(st));
            out_text.release();
            out_text = nb;
            nb.p = nullptr;
            nb.cap = 0;
        }
        cc::k_cc_pack<<<nc, 128, 0, st>>>(ctx->cc_out.as<uint8_t>(), out_cap_off, pack_off,
                                          out_text.as<uint8_t>() + running, nc);
        cc::k_cc_out_off<<<(nc + 256) / 256, 256, 0, st>>>(pack_off, running, d_out_off + a, nc);
        OCB_TRY("cc: pack launch", cudaGetLastError());
        running += tot;
        a = b;
        T.mark("cc: pack");
    }
    OCB_TRY("cc: sync", stream_wait(st));
    *h_total = running;
    return 0;
}

}  // namespace ocb
