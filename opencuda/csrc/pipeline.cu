// The whole compiler on a device-resident batch: preprocess -> lex -> parse
// -> optimize -> emit, with the overflow reruns done on the device too (the
// TUs that outgrew their arena are gathered into a sub-batch, compiled again
// with larger arenas and merged back).  Host work is limited to reading the
// per-TU statuses between passes.
#include <vector>
#include <cub/cub.cuh>
#include "ocb_internal.h"

namespace ocb {

namespace {

// copy TU idx[k] of (src, off) to dst + dst_off[k]; one block per listed TU
__global__ void k_gather_tus(const uint8_t *src, const uint64_t *off, const uint32_t *idx,
                             const uint64_t *dst_off, uint8_t *dst, uint32_t n) {
    uint32_t k = blockIdx.x;
    if (k >= n) return;
    const uint8_t *s = src + off[idx[k]];
    uint8_t *d = dst + dst_off[k];
    uint64_t len = dst_off[k + 1] - dst_off[k];
    for (uint64_t q = threadIdx.x; q < len; q += blockDim.x) d[q] = s[q];
}

// merged lengths/statuses: TU i comes from B (slot ridx[i]) or stays from A
__global__ void k_merge_len(const uint64_t *offA, const int32_t *stA, const uint64_t *offB,
                            const int32_t *stB, const int32_t *ridx, uint32_t n, uint64_t *len,
                            int32_t *stC) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i > n) return;
    if (i == n) {
        len[i] = 0;
        return;
    }
    int32_t k = ridx[i];
    if (k >= 0) {
        len[i] = offB[k + 1] - offB[k];
        stC[i] = stB[k];
    } else {
        len[i] = offA[i + 1] - offA[i];
        stC[i] = stA[i];
    }
}

__global__ void k_merge_copy(const uint8_t *A, const uint64_t *offA, const uint8_t *B,
                             const uint64_t *offB, const int32_t *ridx, const uint64_t *offC,
                             uint8_t *C, uint32_t n) {
    uint32_t i = blockIdx.x;
    if (i >= n) return;
    int32_t k = ridx[i];
    const uint8_t *s = k >= 0 ? B + offB[k] : A + offA[i];
    uint8_t *d = C + offC[i];
    uint64_t len = offC[i + 1] - offC[i];
    for (uint64_t q = threadIdx.x; q < len; q += blockDim.x) d[q] = s[q];
}

struct Part {  // one packed text result: bytes, offsets (n+1), statuses (n)
    DevBuf *text, *off, *status;
};

// Gather the TUs `redo` of `in` (its text and offsets) into ctx->rt_src.
int gather_sub(ocb_ctx *ctx, const uint8_t *d_text, const uint64_t *d_off,
               const std::vector<uint64_t> &h_off, const std::vector<uint32_t> &redo,
               uint64_t *sub_bytes, cudaStream_t st) {
    size_t nr = redo.size();
    std::vector<uint64_t> so(nr + 1, 0);
    for (size_t k = 0; k < nr; ++k) so[k + 1] = so[k] + (h_off[redo[k] + 1] - h_off[redo[k]]);
    OCB_TRY("rerun: text", ctx->rt_src.ensure(so.back() + 64));
    OCB_TRY("rerun: offsets", ctx->rt_src_off.ensure(8 * (nr + 1)));
    OCB_TRY("rerun: index", ctx->rt_idx.ensure(4 * nr + 4));
    OCB_TRY("rerun: h2d", cudaMemcpyAsync(ctx->rt_src_off.p, so.data(), 8 * (nr + 1),
                                          cudaMemcpyHostToDevice, st));
    OCB_TRY("rerun: h2d", cudaMemcpyAsync(ctx->rt_idx.p, redo.data(), 4 * nr,
                                          cudaMemcpyHostToDevice, st));
    k_gather_tus<<<(unsigned)nr, 128, 0, st>>>(d_text, d_off, ctx->rt_idx.as<uint32_t>(),
                                               ctx->rt_src_off.as<uint64_t>(),
                                               ctx->rt_src.as<uint8_t>(), (uint32_t)nr);
    OCB_TRY("rerun: gather", cudaGetLastError());
    *sub_bytes = so.back();
    return 0;
}

// C = A with the TUs of `redo` replaced by B's results (B slot k = redo[k]).
int merge_parts(ocb_ctx *ctx, uint32_t n_tu, Part A, Part B, Part C,
                const std::vector<uint32_t> &redo, uint64_t *h_total, cudaStream_t st) {
    size_t n1 = (size_t)n_tu + 1;
    std::vector<int32_t> ridx(n_tu, -1);
    for (size_t k = 0; k < redo.size(); ++k) ridx[redo[k]] = (int32_t)k;
    OCB_TRY("merge: index", ctx->rt_map.ensure(4 * n1));
    OCB_TRY("merge: lengths", ctx->rt_len.ensure(8 * n1));
    OCB_TRY("merge: offsets", C.off->ensure(8 * n1));
    OCB_TRY("merge: status", C.status->ensure(4 * n1));
    OCB_TRY("merge: h2d", cudaMemcpyAsync(ctx->rt_map.p, ridx.data(), 4 * (size_t)n_tu,
                                          cudaMemcpyHostToDevice, st));
    unsigned g = (unsigned)((n1 + 255) / 256);
    k_merge_len<<<g, 256, 0, st>>>(A.off->as<uint64_t>(), A.status->as<int32_t>(),
                                   B.off->as<uint64_t>(), B.status->as<int32_t>(),
                                   ctx->rt_map.as<int32_t>(), n_tu, ctx->rt_len.as<uint64_t>(),
                                   C.status->as<int32_t>());
    size_t t1 = 0;
    cub::DeviceScan::ExclusiveSum(nullptr, t1, ctx->rt_len.as<uint64_t>(), C.off->as<uint64_t>(),
                                  (int)n1, st);
    OCB_TRY("merge: cub scratch", ctx->cub_tmp.ensure(t1));
    OCB_TRY("merge: scan", cub::DeviceScan::ExclusiveSum(ctx->cub_tmp.p, t1, ctx->rt_len.as<uint64_t>(),
                                                         C.off->as<uint64_t>(), (int)n1, st));
    uint64_t total = 0;
    OCB_TRY("merge: d2h", cudaMemcpyAsync(&total, C.off->as<uint64_t>() + n_tu, 8,
                                          cudaMemcpyDeviceToHost, st));
    OCB_TRY("merge: sync", stream_wait(st));
    OCB_TRY("merge: text", C.text->ensure(total + 64));
    k_merge_copy<<<n_tu, 128, 0, st>>>(A.text->as<uint8_t>(), A.off->as<uint64_t>(),
                                       B.text->as<uint8_t>(), B.off->as<uint64_t>(),
                                       ctx->rt_map.as<int32_t>(), C.off->as<uint64_t>(),
                                       C.text->as<uint8_t>(), n_tu);
    OCB_TRY("merge: copy", cudaGetLastError());
    *h_total = total;
    return 0;
}

void swap_bufs(DevBuf &a, DevBuf &b) {
    DevBuf t = a;
    a = b;
    b = t;
}

}  // namespace

// Run the compiler's back half with arena reruns.  Input: preprocessed text
// (d_text, d_off), statuses so far (d_in_status).  Result: ctx->res_*.
static int cc_with_reruns(ocb_ctx *ctx, const uint8_t *d_text, uint64_t N, const uint64_t *d_off,
                          uint32_t n_tu, const int32_t *d_in_status, int stage,
                          uint64_t *h_total, cudaStream_t st) {
    size_t n1 = (size_t)n_tu + 1;
    OCB_TRY("cc: offsets", ctx->res_off.ensure(8 * n1));
    OCB_TRY("cc: status", ctx->res_status.ensure(4 * n1));
    uint64_t total = 0;
    int rc = cc_device(ctx, d_text, N, d_off, n_tu, d_in_status, stage, 1, ctx->res_text,
                       ctx->res_off.as<uint64_t>(), ctx->res_status.as<int32_t>(), &total, st);
    if (rc) return rc;
    std::vector<int32_t> hs(n_tu), hin(n_tu);
    std::vector<uint64_t> h_off;
    // verdicts of the earlier stages: those TUs keep them and never rerun here
    if (n_tu) OCB_TRY("cc: d2h", cudaMemcpyAsync(hin.data(), d_in_status, 4 * (size_t)n_tu,
                                                 cudaMemcpyDeviceToHost, st));
    for (uint32_t scale = 8; scale <= 64; scale *= 8) {
        if (n_tu) OCB_TRY("cc: d2h", cudaMemcpyAsync(hs.data(), ctx->res_status.p, 4 * (size_t)n_tu,
                                                     cudaMemcpyDeviceToHost, st));
        OCB_TRY("cc: sync", stream_wait(st));
        std::vector<uint32_t> redo;
        for (uint32_t i = 0; i < n_tu; ++i)
            if (hs[i] == OCB_TU_OVERFLOW && hin[i] == 0) redo.push_back(i);
        if (redo.empty()) break;
        if (h_off.empty()) {
            h_off.resize(n1);
            OCB_TRY("cc: d2h", cudaMemcpyAsync(h_off.data(), d_off, 8 * n1, cudaMemcpyDeviceToHost, st));
            OCB_TRY("cc: sync", stream_wait(st));
        }
        uint64_t sub_bytes = 0;
        rc = gather_sub(ctx, d_text, d_off, h_off, redo, &sub_bytes, st);
        if (rc) return rc;
        uint32_t nr = (uint32_t)redo.size();
        OCB_TRY("rerun: status", ctx->rt_in_status.ensure(4 * (size_t)nr + 4));
        OCB_TRY("rerun: status", cudaMemsetAsync(ctx->rt_in_status.p, 0, 4 * (size_t)nr, st));
        OCB_TRY("rerun: offsets", ctx->rt_off.ensure(8 * ((size_t)nr + 1)));
        OCB_TRY("rerun: status", ctx->rt_status.ensure(4 * (size_t)nr + 4));
        uint64_t sub_total = 0;
        rc = cc_device(ctx, ctx->rt_src.as<uint8_t>(), sub_bytes, ctx->rt_src_off.as<uint64_t>(), nr,
                       ctx->rt_in_status.as<int32_t>(), stage, scale, ctx->rt_text,
                       ctx->rt_off.as<uint64_t>(), ctx->rt_status.as<int32_t>(), &sub_total, st);
        if (rc) return rc;
        Part A{&ctx->res_text, &ctx->res_off, &ctx->res_status};
        Part B{&ctx->rt_text, &ctx->rt_off, &ctx->rt_status};
        Part C{&ctx->mg_text, &ctx->mg_off, &ctx->mg_status};
        rc = merge_parts(ctx, n_tu, A, B, C, redo, &total, st);
        if (rc) return rc;
        swap_bufs(ctx->res_text, ctx->mg_text);
        swap_bufs(ctx->res_off, ctx->mg_off);
        swap_bufs(ctx->res_status, ctx->mg_status);
    }
    *h_total = total;
    return 0;
}

// Preprocess with device-side reruns for TUs that outgrew the preprocessor's
// arena.  Result: ctx->pp_text / pp_off / pp_status (and pp_qinc).
int pp_with_reruns(ocb_ctx *ctx, const uint8_t *d_src, uint64_t N, const uint64_t *d_tu_off,
                          uint32_t n_tu, uint64_t *h_total, cudaStream_t st) {
    size_t n1 = (size_t)n_tu + 1;
    OCB_TRY("pp: offsets", ctx->pp_off.ensure(8 * n1));
    OCB_TRY("pp: status", ctx->pp_status.ensure(4 * n1));
    OCB_TRY("pp: flags", ctx->pp_qinc.ensure(4 * n1));
    uint64_t total = 0;
    int rc = pp_device(ctx, d_src, N, d_tu_off, n_tu, 2, ctx->pp_text, ctx->pp_off.as<uint64_t>(),
                       ctx->pp_status.as<int32_t>(), ctx->pp_qinc.as<uint32_t>(), &total, st);
    if (rc) return rc;
    std::vector<int32_t> hs(n_tu);
    std::vector<uint64_t> h_off;
    for (uint32_t scale = 32; scale <= 512; scale *= 16) {
        if (n_tu) OCB_TRY("pp: d2h", cudaMemcpyAsync(hs.data(), ctx->pp_status.p, 4 * (size_t)n_tu,
                                                     cudaMemcpyDeviceToHost, st));
        OCB_TRY("pp: sync", stream_wait(st));
        std::vector<uint32_t> redo;
        for (uint32_t i = 0; i < n_tu; ++i)
            if (hs[i] == OCB_TU_OVERFLOW) redo.push_back(i);
        if (redo.empty()) break;
        if (h_off.empty()) {
            h_off.resize(n1);
            OCB_TRY("pp: d2h", cudaMemcpyAsync(h_off.data(), d_tu_off, 8 * n1, cudaMemcpyDeviceToHost, st));
            OCB_TRY("pp: sync", stream_wait(st));
        }
        uint64_t sub_bytes = 0;
        rc = gather_sub(ctx, d_src, d_tu_off, h_off, redo, &sub_bytes, st);
        if (rc) return rc;
        uint32_t nr = (uint32_t)redo.size();
        OCB_TRY("pp rerun: offsets", ctx->rt_off.ensure(8 * ((size_t)nr + 1)));
        OCB_TRY("pp rerun: status", ctx->rt_status.ensure(4 * (size_t)nr + 4));
        OCB_TRY("pp rerun: flags", ctx->rt_qinc.ensure(4 * (size_t)nr + 4));
        uint64_t sub_total = 0;
        rc = pp_device(ctx, ctx->rt_src.as<uint8_t>(), sub_bytes, ctx->rt_src_off.as<uint64_t>(), nr,
                       scale, ctx->rt_text, ctx->rt_off.as<uint64_t>(), ctx->rt_status.as<int32_t>(),
                       ctx->rt_qinc.as<uint32_t>(), &sub_total, st);
        if (rc) return rc;
        Part A{&ctx->pp_text, &ctx->pp_off, &ctx->pp_status};
        Part B{&ctx->rt_text, &ctx->rt_off, &ctx->rt_status};
        Part C{&ctx->mg_text, &ctx->mg_off, &ctx->mg_status};
        rc = merge_parts(ctx, n_tu, A, B, C, redo, &total, st);
        if (rc) return rc;
        swap_bufs(ctx->pp_text, ctx->mg_text);
        swap_bufs(ctx->pp_off, ctx->mg_off);
        swap_bufs(ctx->pp_status, ctx->mg_status);
        // the include flags of the rerun TUs
        std::vector<uint32_t> qa(n_tu), qb(nr);
        OCB_TRY("pp: d2h", cudaMemcpyAsync(qa.data(), ctx->pp_qinc.p, 4 * (size_t)n_tu, cudaMemcpyDeviceToHost, st));
        OCB_TRY("pp: d2h", cudaMemcpyAsync(qb.data(), ctx->rt_qinc.p, 4 * (size_t)nr, cudaMemcpyDeviceToHost, st));
        OCB_TRY("pp: sync", stream_wait(st));
        for (uint32_t k = 0; k < nr; ++k) qa[redo[k]] = qb[k];
        OCB_TRY("pp: h2d", cudaMemcpyAsync(ctx->pp_qinc.p, qa.data(), 4 * (size_t)n_tu, cudaMemcpyHostToDevice, st));
    }
    *h_total = total;
    return 0;
}

int compile_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t N, const uint64_t *d_tu_off,
                   uint32_t n_tu, int stage, uint64_t *h_total) {
    cudaStream_t st = ctx->stream;
    PhaseTimer T(st);
    if (n_tu == 0) {
        uint64_t z = 0;
        OCB_TRY("pipeline: offsets", ctx->res_off.ensure(8));
        OCB_TRY("pipeline: offsets", ctx->pp_off.ensure(8));
        OCB_TRY("pipeline: status", ctx->res_status.ensure(4));
        OCB_TRY("pipeline: h2d", cudaMemcpyAsync(ctx->res_off.p, &z, 8, cudaMemcpyHostToDevice, st));
        OCB_TRY("pipeline: sync", stream_wait(st));
        *h_total = 0;
        return 0;
    }
    uint64_t pp_total = 0;
    int rc = pp_with_reruns(ctx, d_src, N, d_tu_off, n_tu, &pp_total, st);
    if (rc) return rc;
    T.mark("pipeline: preprocess");
    rc = cc_with_reruns(ctx, ctx->pp_text.as<uint8_t>(), pp_total, ctx->pp_off.as<uint64_t>(), n_tu,
                        ctx->pp_status.as<int32_t>(), stage, h_total, st);
    T.mark("pipeline: compile");
    return rc;
}

}  // namespace ocb
