/*
 * ocb.h -- C ABI of the B200 batch compiler for OpenCUDA's CUDA-C subset.
 *
 * The reference compiler (garrick247/opencuda) is a single-threaded Python
 * program; its only "operator API" is five module functions plus the CLI.
 * This header exports the batch forms of those functions.  Every entry point
 * takes plain pointers and sizes; no exceptions cross the ABI: an `int`
 * return of 0 means success, a negative value an API or CUDA error (text via
 * ocb_last_error), and each translation unit (TU) carries its own status.
 *
 * A batch is one byte buffer holding every TU back to back plus an offset
 * array `tu_off` of n_tu+1 entries: TU i is bytes [tu_off[i], tu_off[i+1]).
 *
 * Threading: one ocb_ctx per (host thread, GPU).  Contexts are independent;
 * sharing one between threads needs external locking.
 */
#ifndef OCB_H
#define OCB_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- per-TU status ------------------------------------------------------ */
#define OCB_TU_OK                 0
/* 1..0xFF: the reference raises on this TU; the value names the class.     */
#define OCB_TU_RAISES_VALUEERROR  1   /* ValueError    (e.g. float.fromhex) */
#define OCB_TU_RAISES_OVERFLOW    2   /* OverflowError (hex float too big)  */
#define OCB_TU_RAISES_PARSEERROR  3   /* opencuda ParseError                */
#define OCB_TU_RAISES_KEYERROR    4
#define OCB_TU_RAISES_REERROR     5   /* re.error from macro templates      */
#define OCB_TU_RAISES_OTHER       6
/* the engine cannot reproduce the reference on this TU                     */
#define OCB_TU_UNSUPPORTED        0x100
/* a per-TU arena was too small                                             */
#define OCB_TU_OVERFLOW           0x200
/* a device loop hit its iteration cap                                      */
#define OCB_TU_TIMEOUT            0x300

/* ---- token record layout (lexer output) --------------------------------- */
/* kindlen = kind << 24 | min(len, 0xFFFFFF).  kind is the numeric value of
 * the reference's TokKind (opencuda/frontend/lexer.py:11-109); a hex-float
 * literal has OCB_TOK_HEXFLOAT or-ed into its kind byte (its reference value
 * is str(float.fromhex(span)), lexer.py:282-284).  start is the byte offset
 * of the token in the batch buffer; line is the reference's Token.line.
 * Each TU's token list ends with an EOF token (kind 88, length 0). */
#define OCB_TOK_HEXFLOAT 0x80
#define OCB_TOK_EOF      88

typedef struct ocb_ctx ocb_ctx;
typedef struct ocb_tokens ocb_tokens;
typedef struct ocb_text ocb_text;

/* Create a context on CUDA device `device`.  flags: reserved, pass 0.
 * Replaces: nothing (the reference keeps no device state). */
int  ocb_create(ocb_ctx **out, int device, uint32_t flags);
void ocb_destroy(ocb_ctx *ctx);
/* Last error text of this context (valid until the next call on it). */
const char *ocb_last_error(ocb_ctx *ctx);
/* Set the `.target` line of the PTX modules that later compiles on this
 * context write (default "sm_120", 1-31 bytes, no control characters).
 * Replaces the CLI's --arch option (opencuda/__main__.py:23-24, written as
 * `.target {arch}` at :64); like the reference, the value is not checked
 * against a list of architectures. */
int  ocb_set_target(ocb_ctx *ctx, const char *arch);
/* Library build string (architecture, version). */
const char *ocb_version(void);

/* ---- lexer -------------------------------------------------------------- */
/* Lex every TU of a host batch.  Replaces opencuda/frontend/lexer.py:258
 * lex(source) -> list[Token], applied to each TU.  Inputs are copied to the
 * device (directly when `src` is pinned); the result holds host copies and is
 * owned by the library until ocb_tokens_free.  TU status is
 * OCB_TU_RAISES_VALUEERROR/OVERFLOW when the reference's lex() raises on a
 * hex float of that TU. */
int  ocb_lex_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off,
                   uint32_t n_tu, ocb_tokens **out);
/* Host views of a token result: arrays of *n_tok entries (tu_tok_off and
 * status: n_tu+1 and n_tu entries). */
int  ocb_tokens_view(const ocb_tokens *t, uint64_t *n_tok,
                     const uint32_t **start, const uint32_t **kindlen,
                     const uint32_t **line, const uint64_t **tu_tok_off,
                     const int32_t **status);
void ocb_tokens_free(ocb_tokens *t);

/* Device-resident form of ocb_lex_batch: every pointer is device memory
 * (d_src 16-byte aligned), the work is queued on `stream` (a cudaStream_t,
 * 0 = the legacy default stream) and the call does not synchronise.  Output
 * arrays hold `tok_cap` tokens (d_line may be NULL); *d_n_tok (device, one
 * uint64) receives the token count.  If the count exceeds tok_cap, no token
 * is written beyond the capacity and the caller re-runs with larger buffers.
 * Scratch memory is owned by the context and reused across calls.
 * Replaces: lexer.py:258 lex(), batched. */
int  ocb_lex_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t n_bytes,
                    const uint64_t *d_tu_off, uint32_t n_tu,
                    uint32_t *d_start, uint32_t *d_kindlen, uint32_t *d_line,
                    uint64_t tok_cap, uint64_t *d_tu_tok_off,
                    int32_t *d_status, uint64_t *d_n_tok, void *stream);

/* ---- preprocessor ------------------------------------------------------- */
/* Preprocess every TU of a host batch.  Replaces
 * opencuda/frontend/preprocess.py:178 preprocess(source, include_paths) as the
 * CLI calls it (__main__.py:39-44) when no quoted include resolves to a file:
 * include lines are blanked, lines spliced, directives and macros applied.
 * The result holds the output text of every TU back to back (off: n_tu+1
 * entries), a per-TU status (OCB_TU_RAISES_REERROR where the reference raises
 * re.error, OCB_TU_UNSUPPORTED / OVERFLOW / TIMEOUT where the engine cannot
 * reproduce it) and a per-TU flag set when a quoted #include line was blanked
 * (a caller with include directories resolves those TUs on the host). */
int  ocb_preprocess_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off,
                          uint32_t n_tu, ocb_text **out);
int  ocb_text_view(const ocb_text *t, uint64_t *n_bytes, const uint8_t **bytes,
                   const uint64_t **off, const int32_t **status,
                   const uint32_t **qinclude);
void ocb_text_free(ocb_text *t);

/* ---- parser ------------------------------------------------------------- */
/* Preprocess, lex and parse every TU of a host batch.  Replaces
 * opencuda/frontend/parser.py:4446 parse(source) applied to the preprocessed
 * text (the CLI's __main__.py:39-51 path up to the IR).  Each TU's output is
 * its IR as canonical text (one line per kernel, parameter, shared/local
 * array, block, instruction and terminator; the line grammar of the oracle's
 * IR dump).  Status per TU: OCB_TU_OK, OCB_TU_RAISES_* where the reference
 * raises (ParseError, ValueError, ...), OCB_TU_UNSUPPORTED for constructs this
 * engine does not reproduce, OCB_TU_OVERFLOW when arena retries ran out.
 * Free the result with ocb_text_free. */
int  ocb_parse_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off,
                     uint32_t n_tu, ocb_text **out);

/* As ocb_parse_batch, then optimize every kernel.  Replaces
 * opencuda/ir/optimize.py:1443 optimize(module) (with the unroller of
 * ir/unroll.py); the text is the optimized IR in the same line format. */
int  ocb_optimize_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off,
                        uint32_t n_tu, ocb_text **out);

/* Preprocess, lex, parse (and, with `optimized`, optimize) every TU, then
 * check its IR with the reference's verifier.  Replaces
 * opencuda/ir/verify_ir.py:302 verify_module(module, check_reachability)
 * (verify_kernel :86-247, dominators of ir/dominator.py:44-112) applied to
 * parse(source) or optimize(parse(source)).  Each TU's text: for every kernel
 * with violations, in module order, a line `kernel <name>` and then one line
 * per error string, in the reference's order and wording; empty when the IR
 * is clean.  Status per TU as for ocb_parse_batch; OCB_TU_UNSUPPORTED also
 * where two or more non-natural-loop errors of one back edge would come out
 * in a Python set's order.  Free the result with ocb_text_free. */
int  ocb_verify_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off,
                      uint32_t n_tu, int optimized, int check_reachability,
                      ocb_text **out);

/* ---- compiler ------------------------------------------------------------ */
/* Compile every TU of a host batch to PTX: preprocess, lex, parse, optimize,
 * allocate registers and emit.  Replaces the CLI path
 * `python -m opencuda X.cu --emit-ptx` (opencuda/__main__.py:36-85:
 * preprocess -> parse -> optimize -> codegen/emit.py:3126 ir_to_ptx -> module
 * text with `.target sm_120`).  Each TU's text is the whole PTX module the CLI
 * would write.  Status per TU as for ocb_parse_batch; a TU where the
 * reference raises during emission (e.g. OverflowError packing a float
 * literal) reports that exception. */
int  ocb_compile_batch(ocb_ctx *ctx, const uint8_t *src, const uint64_t *tu_off,
                       uint32_t n_tu, ocb_text **out);

/* Device-resident form of ocb_parse_batch / ocb_optimize_batch /
 * ocb_compile_batch (stage 0, 1, 2): the batch is already in device memory
 * (d_src, d_tu_off[n_tu+1] as for ocb_lex_device) and the result stays there.
 * TUs that outgrow their arena are gathered, run again with larger arenas and
 * merged back on the device.  On return the work is complete and
 * *d_out / *out_bytes / *d_out_off[n_tu+1] / *d_status[n_tu] describe the
 * packed outputs; they are owned by the context and stay valid until its next
 * call. */
int  ocb_compile_device(ocb_ctx *ctx, const uint8_t *d_src, uint64_t n_bytes,
                        const uint64_t *d_tu_off, uint32_t n_tu, int stage,
                        const uint8_t **d_out, uint64_t *out_bytes,
                        const uint64_t **d_out_off, const int32_t **d_status);

/* Per-kernel timing of the compiler's three kernels, for measurement:
 * ocb_kernel_profile(ctx, 1) zeroes the counters and brackets every later
 * launch of k_cc_parse, k_cc_opt and k_cc_emit with CUDA events on the
 * context's stream (0 turns it off).  ocb_kernel_times fills ms[3] with the
 * summed event durations and launches[3] with the launch counts, in that
 * kernel order. */
int  ocb_kernel_profile(ocb_ctx *ctx, int enable);
/* The context's own CUDA stream (a cudaStream_t), on which every batch call
 * queues its work; for callers that time or order work around those calls. */
void *ocb_stream(ocb_ctx *ctx);
int  ocb_kernel_times(const ocb_ctx *ctx, double *ms, uint64_t *launches);

/* Allocation-free form of ocb_lex_device, for callers that may not allocate
 * device memory when they lex (a framework's memory pool or a fixed arena that
 * forbids cudaMalloc/cudaFree after start-up, or a thread that must not take
 * the allocator's lock).  It needs no context: all scratch lives in one 8 MiB
 * device array inside libocb.so, which every GPU that loads the library holds
 * until the process exits.  Limits: n_bytes <= 4 MiB and n_tu <= 16384;
 * larger batches are rejected with -2 before any work is queued.  Arguments
 * and outputs are those of ocb_lex_device (device pointers, work queued on
 * `stream`, no synchronisation); `err` (may be NULL) receives a message of at
 * most err_len-1 bytes on failure.  The first call on a device (and the first
 * after a device reset) does a set-up with that device current: it uploads the
 * keyword table; every call looks up the array's device address, which does not
 * allocate.  Make that first call before any stream capture.  Every call shares
 * the one array, so calls whose work overlaps on the GPU (other streams, other
 * host threads) race: serialise them.  No counterpart in the reference. */
int  ocb_lex_device_static(const uint8_t *d_src, uint64_t n_bytes,
                           const uint64_t *d_tu_off, uint32_t n_tu,
                           uint32_t *d_start, uint32_t *d_kindlen, uint32_t *d_line,
                           uint64_t tok_cap, uint64_t *d_tu_tok_off,
                           int32_t *d_status, uint64_t *d_n_tok, void *stream,
                           char *err, size_t err_len);

#ifdef __cplusplus
}
#endif

#endif /* OCB_H */
