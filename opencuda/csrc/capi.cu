// C ABI entry points (include/ocb.h): contexts, host-buffer wrappers around
// the device pipelines, result objects.
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>
#include "ocb_internal.h"

PhaseTimer::PhaseTimer(cudaStream_t s) : st(s) {
    const char *v = getenv("OCB_TIMING");
    on = v && *v && *v != '0';
    t0 = 0;
    if (on) mark(nullptr);
}
void PhaseTimer::mark(const char *what) {
    if (!on) return;
    cudaStreamSynchronize(st);
    double t = std::chrono::duration<double, std::milli>(
                   std::chrono::steady_clock::now().time_since_epoch()).count();
    if (what) fprintf(stderr, "[ocb] %-22s %9.2f ms\n", what, t - t0);
    t0 = t;
}

namespace ocb {

int fail(ocb_ctx *ctx, const char *what, cudaError_t e) {
    if (ctx) {
        ctx->err = what;
        ctx->err += ": ";
        ctx->err += cudaGetErrorString(e);
    }
    return -(int)(e ? e : 1);
}

int fail(ocb_ctx *ctx, const std::string &msg) {
    if (ctx) ctx->err = msg;
    return -1;
}

cudaError_t stream_wait(cudaStream_t st) {
    static const double limit_s = [] {
        const char *v = getenv("OCB_WATCHDOG_S");
        double x = v && *v ? atof(v) : 0.0;
        return x > 0 ? x : 1800.0;
    }();
    auto t0 = std::chrono::steady_clock::now();
    for (uint64_t it = 0;; ++it) {
        cudaError_t e = cudaStreamQuery(st);
        if (e != cudaErrorNotReady) return e;
        double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (dt > limit_s) return cudaErrorTimeout;
        if (dt < 0.002) std::this_thread::yield();
        else std::this_thread::sleep_for(std::chrono::microseconds(100));
    }
}

}  // namespace ocb

using namespace ocb;

extern "C" {

const char *ocb_version(void) {
    return "opencuda-b200 0.1 (sm_100a)";
}

int ocb_create(ocb_ctx **out, int device, uint32_t flags) {
    (void)flags;
    if (!out) return -1;
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) return -(int)e;
    if (device < 0 || device >= n) return -1;
    e = cudaSetDevice(device);
    if (e != cudaSuccess) return -(int)e;
    ocb_ctx *ctx = new (std::nothrow) ocb_ctx();
    if (!ctx) return -1;
    ctx->device = device;
    e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete ctx;
        return -(int)e;
    }
    *out = ctx;
    return 0;
}

void ocb_destroy(ocb_ctx *ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    if (ctx->stream) stream_wait(ctx->stream);
    for (DevBuf *b : {&ctx->lex_scratch, &ctx->cub_tmp, &ctx->d_src, &ctx->d_tu_off,
                      &ctx->d_tok_start, &ctx->d_tok_kl, &ctx->d_tok_line, &ctx->d_tu_tok,
                      &ctx->d_status, &ctx->d_count, &ctx->pp_scratch, &ctx->pp_arena,
                      &ctx->pp_text, &ctx->pp_off, &ctx->pp_status, &ctx->pp_qinc,
                      &ctx->cc_tok, &ctx->cc_scratch, &ctx->cc_arena, &ctx->cc_out,
                      &ctx->cc_text, &ctx->cc_off, &ctx->cc_status, &ctx->cc_in_status,
                      &ctx->cc_order, &ctx->cc_spill,
                      &ctx->res_text, &ctx->res_off, &ctx->res_status, &ctx->rt_src,
                      &ctx->rt_src_off, &ctx->rt_idx, &ctx->rt_map, &ctx->rt_len,
                      &ctx->rt_in_status, &ctx->rt_text, &ctx->rt_off, &ctx->rt_status,
                      &ctx->rt_qinc, &ctx->mg_text, &ctx->mg_off, &ctx->mg_status})
        b->release();
    ctx->cc_ptext.release();
    ctx->cc_pmeta.release();
    for (int s = 0; s < ocb_ctx::kCCStreams; ++s) {
        if (ctx->cc_streams[s]) {
            stream_wait(ctx->cc_streams[s]);
            cudaStreamDestroy(ctx->cc_streams[s]);
        }
        ctx->cc_arena_s[s].release();
        ctx->cc_spill_s[s].release();
    }
    ctx->h_stage.release();
    for (cudaEvent_t &e : ctx->kev)
        if (e) cudaEventDestroy(e);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

const char *ocb_last_error(ocb_ctx *ctx) {
    return ctx ? ctx->err.c_str() : "null context";
}

int ocb_set_target(ocb_ctx *ctx, const char *arch) {
    if (!ctx || !arch) return fail(ctx, "ocb_set_target: null argument");
    size_t n = strlen(arch);
    if (n == 0 || n >= sizeof ctx->target)
        return fail(ctx, "ocb_set_target: target must be 1 to 31 bytes");
    for (size_t i = 0; i < n; ++i)
        if ((unsigned char)arch[i] < 0x20 || (unsigned char)arch[i] == 0x7F)
            return fail(ctx, "ocb_set_target: control character in target");
    memcpy(ctx->target, arch, n + 1);
    return 0;
}

int ocb_lex_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t n_bytes, const uint64_t *d_tu_off,
                   uint32_t n_tu, uint32_t *d_start, uint32_t *d_kindlen, uint32_t *d_line,
                   uint64_t tok_cap, uint64_t *d_tu_tok_off, int32_t *d_status, uint64_t *d_n_tok,
                   void *stream) {
    if (!ctx) return -1;
    OCB_TRY("cudaSetDevice", cudaSetDevice(ctx->device));
    return lex_device(ctx, d_src, n_bytes, d_tu_off, n_tu, d_start, d_kindlen, d_line, tok_cap,
                      d_tu_tok_off, d_status, d_n_tok, (cudaStream_t)stream);
}

int ocb_lex_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                  ocb_tokens **out) {
    if (!ctx || !out || !tu_off) return fail(ctx, "ocb_lex_batch: null argument");
    *out = nullptr;
    OCB_TRY("cudaSetDevice", cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    if (tu_off[0] != 0) return fail(ctx, "ocb_lex_batch: tu_off[0] must be 0");
    for (uint32_t i = 0; i < n_tu; ++i)
        if (tu_off[i + 1] < tu_off[i]) return fail(ctx, "ocb_lex_batch: tu_off not monotone");
    uint64_t N = tu_off[n_tu];
    if (N && !src) return fail(ctx, "ocb_lex_batch: null source");
    // host -> device: straight from the caller's buffer when it is pinned,
    // else through the context's pinned staging buffer
    const uint8_t *hs = src;
    cudaPointerAttributes pa;
    if (N && (cudaPointerGetAttributes(&pa, src) != cudaSuccess || pa.type != cudaMemoryTypeHost)) {
        cudaGetLastError();  // clear a failed attribute query
        OCB_TRY("pinned staging", ctx->h_stage.ensure(N));
        memcpy(ctx->h_stage.p, src, N);
        hs = ctx->h_stage.as<uint8_t>();
    }
    OCB_TRY("device source", ctx->d_src.ensure(N + 64));
    OCB_TRY("device offsets", ctx->d_tu_off.ensure(8 * (size_t)(n_tu + 1)));
    if (N) OCB_TRY("h2d source", cudaMemcpyAsync(ctx->d_src.p, hs, N, cudaMemcpyHostToDevice, st));
    OCB_TRY("h2d offsets", cudaMemcpyAsync(ctx->d_tu_off.p, tu_off, 8 * (size_t)(n_tu + 1),
                                           cudaMemcpyHostToDevice, st));
    uint64_t cap = N + n_tu + 1;
    OCB_TRY("device tokens", ctx->d_tok_start.ensure(4 * cap));
    OCB_TRY("device tokens", ctx->d_tok_kl.ensure(4 * cap));
    OCB_TRY("device tokens", ctx->d_tok_line.ensure(4 * cap));
    OCB_TRY("device tu offsets", ctx->d_tu_tok.ensure(8 * (size_t)(n_tu + 1)));
    OCB_TRY("device status", ctx->d_status.ensure(4 * (size_t)n_tu + 4));
    OCB_TRY("device count", ctx->d_count.ensure(8));
    int rc = lex_device(ctx, ctx->d_src.as<uint8_t>(), N, ctx->d_tu_off.as<uint64_t>(), n_tu,
                        ctx->d_tok_start.as<uint32_t>(), ctx->d_tok_kl.as<uint32_t>(),
                        ctx->d_tok_line.as<uint32_t>(), cap, ctx->d_tu_tok.as<uint64_t>(),
                        ctx->d_status.as<int32_t>(), ctx->d_count.as<uint64_t>(), st);
    if (rc) return rc;
    uint64_t n_tok = 0;
    OCB_TRY("d2h count", cudaMemcpyAsync(&n_tok, ctx->d_count.p, 8, cudaMemcpyDeviceToHost, st));
    OCB_TRY("lex sync", stream_wait(st));
    if (n_tok > cap) return fail(ctx, "ocb_lex_batch: token capacity exceeded");
    ocb_tokens *t = new (std::nothrow) ocb_tokens();
    if (!t) return fail(ctx, "ocb_lex_batch: out of host memory");
    t->n_tok = n_tok;
    t->n_tu = n_tu;
    t->start.resize(n_tok);
    t->kindlen.resize(n_tok);
    t->line.resize(n_tok);
    t->tu_tok_off.resize((size_t)n_tu + 1);
    t->status.resize(n_tu);
    cudaError_t e = cudaSuccess;
    if (n_tok) {
        e = cudaMemcpyAsync(t->start.data(), ctx->d_tok_start.p, 4 * n_tok, cudaMemcpyDeviceToHost, st);
        if (!e) e = cudaMemcpyAsync(t->kindlen.data(), ctx->d_tok_kl.p, 4 * n_tok, cudaMemcpyDeviceToHost, st);
        if (!e) e = cudaMemcpyAsync(t->line.data(), ctx->d_tok_line.p, 4 * n_tok, cudaMemcpyDeviceToHost, st);
    }
    if (!e) e = cudaMemcpyAsync(t->tu_tok_off.data(), ctx->d_tu_tok.p, 8 * ((size_t)n_tu + 1),
                                cudaMemcpyDeviceToHost, st);
    if (!e && n_tu) e = cudaMemcpyAsync(t->status.data(), ctx->d_status.p, 4 * (size_t)n_tu,
                                        cudaMemcpyDeviceToHost, st);
    if (!e) e = stream_wait(st);
    if (e) {
        delete t;
        return fail(ctx, "d2h tokens", e);
    }
    *out = t;
    return 0;
}

int ocb_tokens_view(const ocb_tokens *t, uint64_t *n_tok, const uint32_t **start,
                    const uint32_t **kindlen, const uint32_t **line, const uint64_t **tu_tok_off,
                    const int32_t **status) {
    if (!t) return -1;
    if (n_tok) *n_tok = t->n_tok;
    if (start) *start = t->start.data();
    if (kindlen) *kindlen = t->kindlen.data();
    if (line) *line = t->line.data();
    if (tu_tok_off) *tu_tok_off = t->tu_tok_off.data();
    if (status) *status = t->status.data();
    return 0;
}

void ocb_tokens_free(ocb_tokens *t) { delete t; }

// Host batch -> device buffers (source copied through pinned staging when the
// caller's buffer is pageable).
static int upload_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                        uint64_t &N) {
    if (tu_off[0] != 0) return fail(ctx, "tu_off[0] must be 0");
    for (uint32_t i = 0; i < n_tu; ++i)
        if (tu_off[i + 1] < tu_off[i]) return fail(ctx, "tu_off not monotone");
    N = tu_off[n_tu];
    if (N && !src) return fail(ctx, "null source");
    cudaStream_t st = ctx->stream;
    const uint8_t *hs = src;
    cudaPointerAttributes pa;
    if (N && (cudaPointerGetAttributes(&pa, src) != cudaSuccess || pa.type != cudaMemoryTypeHost)) {
        cudaGetLastError();
        OCB_TRY("pinned staging", ctx->h_stage.ensure(N));
        memcpy(ctx->h_stage.p, src, N);
        hs = ctx->h_stage.as<uint8_t>();
    }
    OCB_TRY("device source", ctx->d_src.ensure(N + 64));
    OCB_TRY("device offsets", ctx->d_tu_off.ensure(8 * (size_t)(n_tu + 1)));
    if (N) OCB_TRY("h2d source", cudaMemcpyAsync(ctx->d_src.p, hs, N, cudaMemcpyHostToDevice, st));
    OCB_TRY("h2d offsets", cudaMemcpyAsync(ctx->d_tu_off.p, tu_off, 8 * (size_t)(n_tu + 1),
                                           cudaMemcpyHostToDevice, st));
    return 0;
}

// Device result (text, offsets, statuses, include flags) -> host ocb_text.
static int download_text(ocb_ctx *ctx, ocb_text *t, uint32_t n_tu, uint64_t total,
                         const DevBuf &text, const DevBuf &off, const DevBuf &status) {
    cudaStream_t st = ctx->stream;
    t->n_tu = n_tu;
    t->bytes.resize(total);
    t->off.resize((size_t)n_tu + 1);
    t->status.resize(n_tu);
    t->qinclude.resize(n_tu);
    cudaError_t e = cudaSuccess;
    if (total) e = cudaMemcpyAsync(t->bytes.data(), text.p, total, cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaMemcpyAsync(t->off.data(), off.p, 8 * ((size_t)n_tu + 1),
                                cudaMemcpyDeviceToHost, st);
    if (!e && n_tu) e = cudaMemcpyAsync(t->status.data(), status.p, 4 * (size_t)n_tu,
                                        cudaMemcpyDeviceToHost, st);
    if (!e && n_tu) e = cudaMemcpyAsync(t->qinclude.data(), ctx->pp_qinc.p, 4 * (size_t)n_tu,
                                        cudaMemcpyDeviceToHost, st);
    if (!e) e = stream_wait(st);
    if (e) return fail(ctx, "d2h text", e);
    return 0;
}

int ocb_preprocess_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                         ocb_text **out) {
    if (!ctx || !out || !tu_off) return fail(ctx, "ocb_preprocess_batch: null argument");
    *out = nullptr;
    OCB_TRY("cudaSetDevice", cudaSetDevice(ctx->device));
    uint64_t N = 0;
    int rc = upload_batch(ctx, src, tu_off, n_tu, N);
    if (rc) return rc;
    uint64_t total = 0;
    rc = pp_with_reruns(ctx, ctx->d_src.as<uint8_t>(), N, ctx->d_tu_off.as<uint64_t>(), n_tu,
                        &total, ctx->stream);
    if (rc) return rc;
    ocb_text *t = new (std::nothrow) ocb_text();
    if (!t) return fail(ctx, "ocb_preprocess_batch: out of host memory");
    rc = download_text(ctx, t, n_tu, total, ctx->pp_text, ctx->pp_off, ctx->pp_status);
    if (rc) {
        delete t;
        return rc;
    }
    *out = t;
    return 0;
}

static int stage_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                       int stage, ocb_text **out) {
    if (!ctx || !out || !tu_off) return fail(ctx, "null argument");
    *out = nullptr;
    OCB_TRY("cudaSetDevice", cudaSetDevice(ctx->device));
    PhaseTimer T(ctx->stream);
    uint64_t N = 0;
    int rc = upload_batch(ctx, src, tu_off, n_tu, N);
    if (rc) return rc;
    T.mark("upload");
    uint64_t total = 0;
    rc = compile_device(ctx, ctx->d_src.as<uint8_t>(), N, ctx->d_tu_off.as<uint64_t>(), n_tu,
                        stage, &total);
    if (rc) return rc;
    ocb_text *t = new (std::nothrow) ocb_text();
    if (!t) return fail(ctx, "out of host memory");
    rc = download_text(ctx, t, n_tu, total, ctx->res_text, ctx->res_off, ctx->res_status);
    T.mark("download");
    if (rc) {
        delete t;
        return rc;
    }
    *out = t;
    return 0;
}

int ocb_parse_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                    ocb_text **out) {
    return stage_batch(ctx, src, tu_off, n_tu, 0, out);
}

int ocb_optimize_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                       ocb_text **out) {
    return stage_batch(ctx, src, tu_off, n_tu, 1, out);
}

int ocb_compile_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                      ocb_text **out) {
    return stage_batch(ctx, src, tu_off, n_tu, 2, out);
}

int ocb_verify_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                     int optimized, int check_reachability, ocb_text **out) {
    return stage_batch(ctx, src, tu_off, n_tu, 3 + (optimized ? 1 : 0) + (check_reachability ? 2 : 0),
                       out);
}

int ocb_compile_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t n_bytes,
                       const uint64_t *d_tu_off, uint32_t n_tu, int stage,
                       const uint8_t **d_out, uint64_t *out_bytes, const uint64_t **d_out_off,
                       const int32_t **d_status) {
    if (!ctx) return -1;
    if (stage < 0 || stage > 2) return fail(ctx, "ocb_compile_device: stage must be 0, 1 or 2");
    if (n_tu && (!d_src || !d_tu_off)) return fail(ctx, "ocb_compile_device: null argument");
    OCB_TRY("cudaSetDevice", cudaSetDevice(ctx->device));
    uint64_t total = 0;
    int rc = compile_device(ctx, d_src, n_bytes, d_tu_off, n_tu, stage, &total);
    if (rc) return rc;
    ctx->res_bytes = total;
    ctx->res_n_tu = n_tu;
    if (d_out) *d_out = ctx->res_text.as<uint8_t>();
    if (out_bytes) *out_bytes = total;
    if (d_out_off) *d_out_off = ctx->res_off.as<uint64_t>();
    if (d_status) *d_status = ctx->res_status.as<int32_t>();
    return 0;
}

void *ocb_stream(ocb_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

int ocb_kernel_profile(ocb_ctx *ctx, int enable) {
    if (!ctx) return -1;
    OCB_TRY("cudaSetDevice", cudaSetDevice(ctx->device));
    for (cudaEvent_t &e : ctx->kev)
        if (!e) OCB_TRY("event create", cudaEventCreate(&e));
    ctx->kprof_on = enable != 0;
    for (int k = 0; k < 3; ++k) {
        ctx->kms[k] = 0;
        ctx->kn[k] = 0;
    }
    return 0;
}

int ocb_kernel_times(const ocb_ctx *ctx, double *ms, uint64_t *launches) {
    if (!ctx) return -1;
    for (int k = 0; k < 3; ++k) {
        if (ms) ms[k] = ctx->kms[k];
        if (launches) launches[k] = ctx->kn[k];
    }
    return 0;
}

int ocb_text_view(const ocb_text *t, uint64_t *n_bytes, const uint8_t **bytes,
                  const uint64_t **off, const int32_t **status, const uint32_t **qinclude) {
    if (!t) return -1;
    if (n_bytes) *n_bytes = t->bytes.size();
    if (bytes) *bytes = t->bytes.data();
    if (off) *off = t->off.data();
    if (status) *status = t->status.data();
    if (qinclude) *qinclude = t->qinclude.data();
    return 0;
}

void ocb_text_free(ocb_text *t) { delete t; }

}  // extern "C"
