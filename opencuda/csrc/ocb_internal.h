// Internal host-side declarations shared by the library's translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <string>
#include <vector>
#include "../../include/ocb.h"

namespace ocb {

// Grow-only device allocation owned by a context.
struct DevBuf {
    void *p = nullptr;
    size_t cap = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap && p) return cudaSuccess;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        size_t want = bytes < 256 ? 256 : bytes;
        cudaError_t e = cudaMalloc(&p, want);
        if (e == cudaSuccess) cap = want;
        return e;
    }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
    }
    template <class T> T *as() const { return static_cast<T *>(p); }
};

// Grow-only pinned host allocation.
struct HostBuf {
    void *p = nullptr;
    size_t cap = 0;
    cudaError_t ensure(size_t bytes) {
        if (bytes <= cap && p) return cudaSuccess;
        if (p) cudaFreeHost(p);
        p = nullptr;
        cap = 0;
        size_t want = bytes < 256 ? 256 : bytes;
        cudaError_t e = cudaMallocHost(&p, want);
        if (e == cudaSuccess) cap = want;
        return e;
    }
    void release() {
        if (p) cudaFreeHost(p);
        p = nullptr;
        cap = 0;
    }
    template <class T> T *as() const { return static_cast<T *>(p); }
};

}  // namespace ocb

struct ocb_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    // `.target` of the PTX modules this context writes (ocb_set_target)
    char target[32] = "sm_120";
    // lexer scratch
    ocb::DevBuf lex_scratch, cub_tmp;
    // staging for host-buffer entry points
    ocb::DevBuf d_src, d_tu_off, d_tok_start, d_tok_kl, d_tok_line, d_tu_tok,
        d_status, d_count;
    ocb::HostBuf h_stage;
    bool kw_ready = false;
    // preprocessor scratch and outputs
    ocb::DevBuf pp_scratch, pp_arena, pp_text, pp_off, pp_status, pp_qinc;
    // compiler back half (tokens -> IR -> PTX) scratch and outputs
    ocb::DevBuf cc_tok, cc_scratch, cc_arena, cc_out, cc_text, cc_off, cc_status, cc_in_status;
    // compiler: per-chunk TU order (largest first) and the shared spill pool
    ocb::DevBuf cc_order, cc_spill;
    // compiler: the batch gathered largest first (text, offsets, permutation,
    // statuses and lengths in that order) and the chunk streams, each with
    // its own arena and spill pool
    static constexpr int kCCStreams = 4;
    ocb::DevBuf cc_ptext, cc_pmeta;
    cudaStream_t cc_streams[kCCStreams] = {};
    ocb::DevBuf cc_arena_s[kCCStreams], cc_spill_s[kCCStreams];
    // whole-pipeline result (res_*), rerun sub-batches (rt_*) and merge targets (mg_*)
    ocb::DevBuf res_text, res_off, res_status;
    ocb::DevBuf rt_src, rt_src_off, rt_idx, rt_map, rt_len, rt_in_status, rt_text, rt_off,
        rt_status, rt_qinc;
    ocb::DevBuf mg_text, mg_off, mg_status;
    uint64_t res_bytes = 0;
    uint32_t res_n_tu = 0;
    // per-kernel CUDA-event timing of the compiler kernels (ocb_kernel_profile)
    bool kprof_on = false;
    cudaEvent_t kev[4] = {};
    double kms[3] = {};
    uint64_t kn[3] = {};
};

struct ocb_text {
    uint32_t n_tu = 0;
    std::vector<uint8_t> bytes;
    std::vector<uint64_t> off;
    std::vector<int32_t> status;
    std::vector<uint32_t> qinclude;
};

struct ocb_tokens {
    uint64_t n_tok = 0;
    uint32_t n_tu = 0;
    std::vector<uint32_t> start, kindlen, line;
    std::vector<uint64_t> tu_tok_off;
    std::vector<int32_t> status;
};

namespace ocb {
int fail(ocb_ctx *ctx, const char *what, cudaError_t e);
int fail(ocb_ctx *ctx, const std::string &msg);

// Lexer pipeline on device buffers (lex.cu).
int lex_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t n_bytes,
               const uint64_t *d_tu_off, uint32_t n_tu, uint32_t *d_start,
               uint32_t *d_kindlen, uint32_t *d_line, uint64_t tok_cap,
               uint64_t *d_tu_tok_off, int32_t *d_status, uint64_t *d_n_tok,
               cudaStream_t stream);
// Preprocessor on device buffers (pp.cu): output text packed into `out_text`
// (grown as needed) at d_out_off[n_tu+1]; total bytes returned in *h_total.
int pp_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t N, const uint64_t *d_tu_off,
              uint32_t n_tu, uint32_t scale, DevBuf &out_text, uint64_t *d_out_off,
              int32_t *d_status, uint32_t *d_qinc, uint64_t *h_total, cudaStream_t st);
// Back half on device buffers (cc.cu): lex the preprocessed text of each TU,
// parse (and optimize) it and write the TU's IR text into `out_text` at d_out_off[n_tu+1].
// d_in_status holds the earlier stages' verdicts; d_status gets the final ones.
// `stage`: 0 = IR after parse(), 1 = IR after optimize().
int cc_device(ocb_ctx *ctx, const uint8_t *d_text, uint64_t N, const uint64_t *d_off,
              uint32_t n_tu, const int32_t *d_in_status, int stage, uint32_t scale,
              DevBuf &out_text, uint64_t *d_out_off, int32_t *d_status, uint64_t *h_total,
              cudaStream_t st);
// Preprocess with reruns of the TUs that outgrew the preprocessor's arena
// (pipeline.cu).  Result in ctx->pp_text / pp_off / pp_status / pp_qinc.
int pp_with_reruns(ocb_ctx *ctx, const uint8_t *d_src, uint64_t N, const uint64_t *d_tu_off,
                   uint32_t n_tu, uint64_t *h_total, cudaStream_t st);
// The whole pipeline on device buffers (pipeline.cu): preprocess, then
// lex/parse/optimize/emit up to `stage`, with arena reruns on the device.
// Result in ctx->res_text / res_off / res_status (+ ctx->pp_qinc).
int compile_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t N, const uint64_t *d_tu_off,
                   uint32_t n_tu, int stage, uint64_t *h_total);
}  // namespace ocb

// Waits until the work queued on `st` is done, like cudaStreamSynchronize,
// but gives up after the watchdog limit (OCB_WATCHDOG_S seconds in the
// environment, default 1800) and returns cudaErrorTimeout: a host thread
// never blocks forever on a device that stopped making progress.  Polls
// cudaStreamQuery (yielding for the first 2 ms, then sleeping 100 us).
namespace ocb {
cudaError_t stream_wait(cudaStream_t st);
}  // namespace ocb

// Phase timing for tuning: with OCB_TIMING set in the environment, mark()
// synchronises the stream and prints the time since the previous mark.
struct PhaseTimer {
    bool on;
    double t0;
    cudaStream_t st;
    explicit PhaseTimer(cudaStream_t s);
    void mark(const char *what);
};

#define OCB_TRY(what, expr)                                    \
    do {                                                       \
        cudaError_t e_ = (expr);                               \
        if (e_ != cudaSuccess) return ocb::fail(ctx, what, e_); \
    } while (0)
