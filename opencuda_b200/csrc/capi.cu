// C ABI entry points (include/ocb.h): contexts, host-buffer wrappers around
// the device pipelines, result objects.
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
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
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (DevBuf *b : {&ctx->lex_scratch, &ctx->cub_tmp, &ctx->d_src, &ctx->d_tu_off,
                      &ctx->d_tok_start, &ctx->d_tok_kl, &ctx->d_tok_line, &ctx->d_tu_tok,
                      &ctx->d_status, &ctx->d_count, &ctx->pp_scratch, &ctx->pp_arena,
                      &ctx->pp_text, &ctx->pp_off, &ctx->pp_status, &ctx->pp_qinc})
        b->release();
    ctx->h_stage.release();
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
}

const char *ocb_last_error(ocb_ctx *ctx) {
    return ctx ? ctx->err.c_str() : "null context";
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
    OCB_TRY("lex sync", cudaStreamSynchronize(st));
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
    if (!e) e = cudaStreamSynchronize(st);
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

static int download_text(ocb_ctx *ctx, ocb_text *t, uint32_t n_tu, uint64_t total) {
    cudaStream_t st = ctx->stream;
    t->n_tu = n_tu;
    t->bytes.resize(total);
    t->off.resize((size_t)n_tu + 1);
    t->status.resize(n_tu);
    t->qinclude.resize(n_tu);
    cudaError_t e = cudaSuccess;
    if (total) e = cudaMemcpyAsync(t->bytes.data(), ctx->pp_text.p, total, cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaMemcpyAsync(t->off.data(), ctx->pp_off.p, 8 * ((size_t)n_tu + 1),
                                cudaMemcpyDeviceToHost, st);
    if (!e && n_tu) e = cudaMemcpyAsync(t->status.data(), ctx->pp_status.p, 4 * (size_t)n_tu,
                                        cudaMemcpyDeviceToHost, st);
    if (!e && n_tu) e = cudaMemcpyAsync(t->qinclude.data(), ctx->pp_qinc.p, 4 * (size_t)n_tu,
                                        cudaMemcpyDeviceToHost, st);
    if (!e) e = cudaStreamSynchronize(st);
    if (e) return fail(ctx, "d2h text", e);
    return 0;
}

int ocb_preprocess_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                         ocb_text **out) {
    if (!ctx || !out || !tu_off) return fail(ctx, "ocb_preprocess_batch: null argument");
    *out = nullptr;
    OCB_TRY("cudaSetDevice", cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    uint64_t N = 0;
    int rc = upload_batch(ctx, src, tu_off, n_tu, N);
    if (rc) return rc;
    OCB_TRY("device offsets", ctx->pp_off.ensure(8 * ((size_t)n_tu + 1)));
    OCB_TRY("device status", ctx->pp_status.ensure(4 * (size_t)n_tu + 4));
    OCB_TRY("device flags", ctx->pp_qinc.ensure(4 * (size_t)n_tu + 4));
    uint64_t total = 0;
    rc = pp_device(ctx, ctx->d_src.as<uint8_t>(), N, ctx->d_tu_off.as<uint64_t>(), n_tu, 2,
                   ctx->pp_text, ctx->pp_off.as<uint64_t>(), ctx->pp_status.as<int32_t>(),
                   ctx->pp_qinc.as<uint32_t>(), &total, st);
    if (rc) return rc;
    ocb_text *t = new (std::nothrow) ocb_text();
    if (!t) return fail(ctx, "ocb_preprocess_batch: out of host memory");
    rc = download_text(ctx, t, n_tu, total);
    if (rc) {
        delete t;
        return rc;
    }
    // TUs whose arena was too small (macro growth) run again, alone, with a
    // larger arena; their output replaces the first attempt's.
    for (uint32_t scale = 32; scale <= 512; scale *= 16) {
        std::vector<uint32_t> redo;
        for (uint32_t i = 0; i < n_tu; ++i)
            if (t->status[i] == OCB_TU_OVERFLOW) redo.push_back(i);
        if (redo.empty()) break;
        std::vector<uint64_t> sub_off(redo.size() + 1, 0);
        for (size_t k = 0; k < redo.size(); ++k)
            sub_off[k + 1] = sub_off[k] + (tu_off[redo[k] + 1] - tu_off[redo[k]]);
        std::vector<uint8_t> sub(sub_off.back() + 1);
        for (size_t k = 0; k < redo.size(); ++k)
            memcpy(sub.data() + sub_off[k], src + tu_off[redo[k]], sub_off[k + 1] - sub_off[k]);
        uint64_t sN = 0;
        rc = upload_batch(ctx, sub.data(), sub_off.data(), (uint32_t)redo.size(), sN);
        uint64_t stotal = 0;
        if (!rc)
            rc = pp_device(ctx, ctx->d_src.as<uint8_t>(), sN, ctx->d_tu_off.as<uint64_t>(),
                           (uint32_t)redo.size(), scale, ctx->pp_text, ctx->pp_off.as<uint64_t>(),
                           ctx->pp_status.as<int32_t>(), ctx->pp_qinc.as<uint32_t>(), &stotal, st);
        ocb_text r;
        if (!rc) rc = download_text(ctx, &r, (uint32_t)redo.size(), stotal);
        if (rc) {
            delete t;
            return rc;
        }
        // splice the retried TUs into the result
        ocb_text m;
        m.n_tu = n_tu;
        m.off.resize((size_t)n_tu + 1);
        m.status = t->status;
        m.qinclude = t->qinclude;
        size_t k = 0;
        for (uint32_t i = 0; i < n_tu; ++i) {
            m.off[i] = m.bytes.size();
            if (k < redo.size() && redo[k] == i) {
                m.bytes.insert(m.bytes.end(), r.bytes.begin() + r.off[k], r.bytes.begin() + r.off[k + 1]);
                m.status[i] = r.status[k];
                m.qinclude[i] = r.qinclude[k];
                ++k;
            } else {
                m.bytes.insert(m.bytes.end(), t->bytes.begin() + t->off[i], t->bytes.begin() + t->off[i + 1]);
            }
        }
        m.off[n_tu] = m.bytes.size();
        *t = std::move(m);
    }
    *out = t;
    return 0;
}

// Run the back half (lex + parse) over TUs already preprocessed on the host;
// TUs that outgrow their arena run again alone with larger arenas.
static int compile_text(ocb_ctx *ctx, const ocb_text &pp, int stage, ocb_text *out) {
    cudaStream_t st = ctx->stream;
    uint32_t n_tu = pp.n_tu;
    out->n_tu = n_tu;
    out->status.assign(n_tu, 0);
    out->qinclude = pp.qinclude;
    out->off.assign((size_t)n_tu + 1, 0);
    out->bytes.clear();
    std::vector<uint32_t> todo(n_tu);
    for (uint32_t i = 0; i < n_tu; ++i) todo[i] = i;
    std::vector<std::vector<uint8_t>> res(n_tu);
    PhaseTimer T(st);
    for (uint32_t scale = 1; !todo.empty(); scale *= 8) {
        // sub-batch of the pending TUs
        std::vector<uint64_t> off(todo.size() + 1, 0);
        for (size_t k = 0; k < todo.size(); ++k)
            off[k + 1] = off[k] + (pp.off[todo[k] + 1] - pp.off[todo[k]]);
        std::vector<uint8_t> text(off.back() + 1);
        std::vector<int32_t> in_st(todo.size());
        for (size_t k = 0; k < todo.size(); ++k) {
            memcpy(text.data() + off[k], pp.bytes.data() + pp.off[todo[k]], off[k + 1] - off[k]);
            in_st[k] = pp.status[todo[k]];
        }
        uint64_t N = 0;
        int rc = upload_batch(ctx, text.data(), off.data(), (uint32_t)todo.size(), N);
        if (rc) return rc;
        size_t nt = todo.size();
        OCB_TRY("device status", ctx->cc_in_status.ensure(4 * nt + 4));
        OCB_TRY("device status", ctx->cc_status.ensure(4 * nt + 4));
        OCB_TRY("device offsets", ctx->cc_off.ensure(8 * (nt + 1)));
        OCB_TRY("h2d status", cudaMemcpyAsync(ctx->cc_in_status.p, in_st.data(), 4 * nt,
                                              cudaMemcpyHostToDevice, st));
        uint64_t total = 0;
        T.mark(scale == 1 ? "cc: upload" : "cc: upload (retry)");
        rc = cc_device(ctx, ctx->d_src.as<uint8_t>(), N, ctx->d_tu_off.as<uint64_t>(),
                       (uint32_t)nt, ctx->cc_in_status.as<int32_t>(), stage, scale, ctx->cc_text,
                       ctx->cc_off.as<uint64_t>(), ctx->cc_status.as<int32_t>(), &total, st);
        if (rc) return rc;
        std::vector<uint8_t> bytes(total);
        std::vector<uint64_t> o(nt + 1);
        std::vector<int32_t> s(nt);
        cudaError_t e = cudaSuccess;
        if (total) e = cudaMemcpyAsync(bytes.data(), ctx->cc_text.p, total, cudaMemcpyDeviceToHost, st);
        if (!e) e = cudaMemcpyAsync(o.data(), ctx->cc_off.p, 8 * (nt + 1), cudaMemcpyDeviceToHost, st);
        if (!e) e = cudaMemcpyAsync(s.data(), ctx->cc_status.p, 4 * nt, cudaMemcpyDeviceToHost, st);
        if (!e) e = cudaStreamSynchronize(st);
        if (e) return fail(ctx, "d2h compile output", e);
        T.mark("cc: download");
        std::vector<uint32_t> next;
        for (size_t k = 0; k < nt; ++k) {
            uint32_t i = todo[k];
            out->status[i] = s[k];
            if (s[k] == OCB_TU_OVERFLOW && scale < 64) next.push_back(i);
            else res[i].assign(bytes.begin() + o[k], bytes.begin() + o[k + 1]);
        }
        todo.swap(next);
    }
    for (uint32_t i = 0; i < n_tu; ++i) {
        out->off[i] = out->bytes.size();
        out->bytes.insert(out->bytes.end(), res[i].begin(), res[i].end());
    }
    out->off[n_tu] = out->bytes.size();
    return 0;
}

static int stage_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                       int stage, ocb_text **out) {
    if (!ctx || !out || !tu_off) return fail(ctx, "null argument");
    *out = nullptr;
    ocb_text *pp = nullptr;
    PhaseTimer T(ctx->stream);
    int rc = ocb_preprocess_batch(ctx, src, tu_off, n_tu, &pp);
    if (rc) return rc;
    T.mark("preprocess (host api)");
    ocb_text *t = new (std::nothrow) ocb_text();
    if (!t) {
        delete pp;
        return fail(ctx, "out of host memory");
    }
    rc = compile_text(ctx, *pp, stage, t);
    delete pp;
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
