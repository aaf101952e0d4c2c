// Batch lexer kernels for sm_100a (host driver in lex.cu).
//
// Restates opencuda/frontend/lexer.py:258-295 (lex) for every TU of a batch at
// once.  Pipeline over 32-byte windows (one thread each):
//   1. k_lex_map    - transition map of the 8-state mode automaton over the
//                     window (right-to-left composition, 2 byte-permutes per
//                     byte), reset to CODE at TU starts.
//   2. scan(compose)- mode state at every window start.
//   3. k_lex_sync   - from the known state: newlines the reference counts
//                     (segmented by TU) and the window's first sync point (a
//                     position the reference provably starts a token at).
//   4. scans        - segmented newline prefix -> line at each sync point;
//                     suffix-min of sync points -> each thread's segment.
//   5. k_lex_tokens - exact sequential matching of the thread's segment
//                     [S_t, S_t+1), counting (pass A) then writing (pass B).
#pragma once
#include <stdint.h>
#include <string.h>
#include "../../include/ocb.h"
#include "lex_dfa.cuh"
#include "lex_tokdfa.cuh"

namespace ocb {
namespace lex {

constexpr int WIN = 32;          // bytes per thread window
constexpr int LOOK = 4;          // lookahead bytes loaded beyond the window
constexpr int NWORD = (WIN + LOOK) / 4;
constexpr int BLOCK = 256;
constexpr uint64_t NO_SYNC = ~0ull;

__constant__ uint32_t c_tsel[C_NCLS] = OCB_TSEL_INIT;
__device__ KwEntry g_kw[128];

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------
// first i in [0, n) with a[i] >= x (n if none)
__device__ __forceinline__ uint32_t lower_bound_u64(const uint64_t *a, uint32_t n, uint64_t x) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        uint32_t mid = (lo + hi) >> 1;
        if (__ldg(a + mid) < x) lo = mid + 1; else hi = mid;
    }
    return lo;
}
// first i in [0, n) with a[i] > x (n if none)
__device__ __forceinline__ uint32_t upper_bound_u64(const uint64_t *a, uint32_t n, uint64_t x) {
    uint32_t lo = 0, hi = n;
    while (lo < hi) {
        uint32_t mid = (lo + hi) >> 1;
        if (__ldg(a + mid) <= x) lo = mid + 1; else hi = mid;
    }
    return lo;
}

// Bits j in [0, 40) of the span starting at `base`: tus = base+j starts a TU
// that holds bytes; bnd = base+j is any TU boundary (batch end included).
__device__ __forceinline__ void window_masks(const uint64_t *tu_off, uint32_t n_tu, uint64_t N,
                                             uint64_t base, uint64_t &tus, uint64_t &bnd) {
    tus = 0;
    bnd = 0;
    uint32_t k = lower_bound_u64(tu_off, n_tu + 1, base);
    for (; k <= n_tu; ++k) {
        uint64_t x = __ldg(tu_off + k);
        if (x >= base + 40) break;
        uint64_t bit = 1ull << (x - base);
        bnd |= bit;
        if (k < n_tu && x < N) tus |= bit;
    }
}

// Window bytes [base, base+WIN+LOOK) as little-endian words; zero past N.
__device__ __forceinline__ void load_window(const uint8_t *src, uint64_t N, uint64_t base,
                                            uint32_t (&wd)[NWORD]) {
    if (base + WIN + LOOK <= N) {
        const uint4 *v = reinterpret_cast<const uint4 *>(src + base);
        uint4 a = __ldg(v), b = __ldg(v + 1);
        wd[0] = a.x; wd[1] = a.y; wd[2] = a.z; wd[3] = a.w;
        wd[4] = b.x; wd[5] = b.y; wd[6] = b.z; wd[7] = b.w;
        wd[8] = __ldg(reinterpret_cast<const uint32_t *>(src + base + WIN));
    } else {
#pragma unroll
        for (int j = 0; j < NWORD; ++j) {
            uint32_t w = 0;
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                uint64_t q = base + 4 * j + b;
                uint32_t c = q < N ? (uint32_t)__ldg(src + q) : 0u;
                w |= c << (8 * b);
            }
            wd[j] = w;
        }
    }
}
#define WB(i) ((wd[(i) >> 2] >> (8 * ((i) & 3))) & 0xFFu)

// Parity of the backslash run ending right before position q.  Only a quote
// inside a string needs it, and such a run never extends before the string's
// opening quote, so the walk stops at the first non-backslash byte.
__device__ __noinline__ int backslash_run_odd(const uint8_t *src, uint64_t q) {
    int odd = 0;
    while (q > 0 && __ldg(src + q - 1) == '\\') {
        odd ^= 1;
        --q;
    }
    return odd;
}

// Class of window byte I (a compile-time index).
template <int I>
__device__ __forceinline__ uint32_t class_at(const uint32_t (&wd)[NWORD], uint64_t bnd,
                                             const uint8_t *src, uint64_t base) {
    uint32_t c = WB(I);
    if (c != '\n' && c != '/' && c != '*' && c != '\'' && c != '"') return C_OTHER;
    int nv = ((bnd >> (I + 1)) & 1) ? 0 : ((bnd >> (I + 2)) & 1) ? 1 : ((bnd >> (I + 3)) & 1) ? 2 : 3;
    int odd = 0;
    if (c == '"') {
        if (I == 0 || WB(I == 0 ? 0 : I - 1) == '\\') odd = backslash_run_odd(src, base + I);
    }
    return classify(c, WB(I + 1), WB(I + 2), WB(I + 3), nv, odd);
}

template <int I>
struct MapStep {
    static __device__ __forceinline__ void run(const uint32_t (&wd)[NWORD], uint64_t bnd,
                                               uint64_t tus, const uint8_t *src, uint64_t base,
                                               uint64_t N, uint32_t &mlo, uint32_t &mhi) {
        if (base + I < N) {
            uint32_t sel = c_tsel[class_at<I>(wd, bnd, src, base)];
            uint32_t nlo = __byte_perm(mlo, mhi, sel & 0xFFFFu);
            uint32_t nhi = __byte_perm(mlo, mhi, sel >> 16);
            mlo = nlo;
            mhi = nhi;
            if ((tus >> I) & 1) {
                uint32_t v = (mlo & 0xFFu) * 0x01010101u;
                mlo = v;
                mhi = v;
            }
        }
        MapStep<I - 1>::run(wd, bnd, tus, src, base, N, mlo, mhi);
    }
};
template <>
struct MapStep<-1> {
    static __device__ __forceinline__ void run(const uint32_t (&)[NWORD], uint64_t, uint64_t,
                                               const uint8_t *, uint64_t, uint64_t, uint32_t &,
                                               uint32_t &) {}
};

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(BLOCK)
k_lex_map(const uint8_t *__restrict__ src, uint64_t N, const uint64_t *__restrict__ tu_off,
          uint32_t n_tu, uint64_t n_win, uint64_t *__restrict__ maps) {
    uint64_t w = (uint64_t)blockIdx.x * BLOCK + threadIdx.x;
    if (w >= n_win) return;
    uint64_t base = w * WIN;
    uint32_t wd[NWORD];
    load_window(src, N, base, wd);
    uint64_t tus, bnd;
    window_masks(tu_off, n_tu, N, base, tus, bnd);
    uint32_t mlo = 0x03020100u, mhi = 0x07060504u;
    MapStep<WIN - 1>::run(wd, bnd, tus, src, base, N, mlo, mhi);
    maps[w] = ((uint64_t)mhi << 32) | mlo;
}

// Segmented newline record: bit 63 = a TU starts inside, low bits = count.
constexpr uint64_t SEG_FLAG = 1ull << 63;

template <int I>
struct SyncStep {
    static __device__ __forceinline__ void run(const uint32_t (&wd)[NWORD], uint64_t bnd,
                                               uint64_t tus, const uint8_t *src, uint64_t base,
                                               uint64_t N, uint32_t &st, uint64_t &nl, bool &flag,
                                               uint64_t &fsync, uint32_t &sinfo) {
        if (base + I < N) {
            if ((tus >> I) & 1) {
                st = S_CODE;
                nl = 0;
                flag = true;
                if (fsync == NO_SYNC) {
                    fsync = base + I;
                    sinfo = 0x80000000u;
                }
            }
            uint32_t c = WB(I);
            // a newline the reference counts: NEWLINE token, or inside a comment
            if (c == '\n' && st <= S_BC) nl++;
            uint32_t cls = class_at<I>(wd, bnd, src, base);
            if (fsync == NO_SYNC &&
                ((st == S_CODE && (c == ' ' || c == '\t' || c == '\r' || c == '\n')) ||
                 (st == S_LC && c == '\n'))) {
                fsync = base + I + 1;
                sinfo = (uint32_t)nl | (((tus >> (I + 1)) & 1) ? 0x80000000u : 0u);
            }
            st = next_state(c_tsel[cls], st);
        }
        SyncStep<I + 1>::run(wd, bnd, tus, src, base, N, st, nl, flag, fsync, sinfo);
    }
};
template <>
struct SyncStep<WIN> {
    static __device__ __forceinline__ void run(const uint32_t (&)[NWORD], uint64_t, uint64_t,
                                               const uint8_t *, uint64_t, uint64_t, uint32_t &,
                                               uint64_t &, bool &, uint64_t &, uint32_t &) {}
};

__global__ void __launch_bounds__(BLOCK)
k_lex_sync(const uint8_t *__restrict__ src, uint64_t N, const uint64_t *__restrict__ tu_off,
           uint32_t n_tu, uint64_t n_win, const uint64_t *__restrict__ mapscan,
           uint64_t *__restrict__ nlseg, uint64_t *__restrict__ fsync_out,
           uint32_t *__restrict__ sinfo_out) {
    uint64_t w = (uint64_t)blockIdx.x * BLOCK + threadIdx.x;
    if (w >= n_win) return;
    uint64_t base = w * WIN;
    uint32_t wd[NWORD];
    load_window(src, N, base, wd);
    uint64_t tus, bnd;
    window_masks(tu_off, n_tu, N, base, tus, bnd);
    uint32_t st = w == 0 ? S_CODE : (uint32_t)(mapscan[w - 1] & 0xFFu);
    uint64_t nl = 0, fsync = NO_SYNC;
    bool flag = false;
    uint32_t sinfo = 0;
    SyncStep<0>::run(wd, bnd, tus, src, base, N, st, nl, flag, fsync, sinfo);
    nlseg[w] = (flag ? SEG_FLAG : 0) | nl;
    fsync_out[w] = fsync;
    sinfo_out[w] = sinfo;
}

// ---------------------------------------------------------------------------
// sequential matcher
// ---------------------------------------------------------------------------
// Verdict of float.fromhex on a hex-float token (lexer.py:282-284):
// 0 ok, 1 ValueError (no digit either side of the point), 2 OverflowError
// (the value rounds, half to even at 53 bits, to 2**1024 or more).
template <class S>
__device__ __noinline__ uint32_t hexfloat_verdict(S s, uint64_t p, uint64_t n) {
    uint64_t q = p + 2, end = p + n, i0 = q;
    while (q < end && is_hex(s[q])) q++;
    uint64_t ni = q - i0, f0 = q, nf = 0;
    if (q < end && s[q] == '.') {
        q++;
        f0 = q;
        while (q < end && is_hex(s[q])) q++;
        nf = q - f0;
    }
    if (ni == 0 && nf == 0) return 1;
    q++;  // the exponent letter
    bool neg = false;
    if (q < end && (s[q] == '+' || s[q] == '-')) {
        neg = s[q] == '-';
        q++;
    }
    int64_t E = 0;
    while (q < end && is_dig(s[q])) {
        if (E < 100000000) E = E * 10 + (s[q] - '0');
        q++;
    }
    if (neg) E = -E;
    uint64_t nd = ni + nf;
    auto dig = [&](uint64_t k) -> uint32_t {
        uint32_t c = k < ni ? s[i0 + k] : s[f0 + (k - ni)];
        return c <= '9' ? c - '0' : (c | 0x20u) - 'a' + 10;
    };
    int64_t lead = -1;
    for (uint64_t k = 0; k < nd; ++k)
        if (dig(k)) { lead = (int64_t)k; break; }
    if (lead < 0) return 0;
    uint32_t v0 = dig((uint64_t)lead);
    int bl = 32 - __clz(v0);
    int64_t e2 = 4 * ((int64_t)ni - 1 - lead) + (bl - 1) + E;
    if (e2 < 1023) return 0;
    if (e2 > 1023) return 2;
    // exactly at the top binade: overflow iff the 54 leading bits are all one
    int bits = 0;
    for (uint64_t k = (uint64_t)lead; k < nd && bits < 54; ++k) {
        uint32_t v = dig(k);
        int nb = k == (uint64_t)lead ? bl : 4;
        for (int b = nb - 1; b >= 0 && bits < 54; --b, ++bits)
            if (!((v >> b) & 1)) return 0;
    }
    return bits >= 54 ? 2 : 0;
}

template <class S>
__device__ __forceinline__ uint64_t match_hexfloat(S s, uint64_t p, uint64_t e) {
    if (p + 1 >= e || s[p] != '0' || (s[p + 1] | 0x20u) != 'x') return 0;
    uint64_t q = p + 2, h = run_hex(s, q, e);
    if (q + h < e && s[q + h] == '.') {
        uint64_t r = q + h + 1;
        r += run_hex(s, r, e);
        uint64_t x = match_exp(s, r, e, 'p');
        if (x) return r + x + opt_fFlL(s, r + x, e) - p;
    }
    if (h) {
        uint64_t r = q + h, x = match_exp(s, r, e, 'p');
        if (x) return r + x + opt_fFlL(s, r + x, e) - p;
    }
    return 0;
}

template <class S>
__device__ __forceinline__ uint64_t match_float(S s, uint64_t p, uint64_t e) {
    uint64_t d = run_digits(s, p, e);
    bool dot = p + d < e && s[p + d] == '.';
    if (dot) {
        uint64_t r = p + d + 1, f = run_digits(s, r, e);
        if (d || f) {  // [0-9]+\.[0-9]*  or  [0-9]*\.[0-9]+
            r += f;
            r += match_exp(s, r, e, 'e');
            return r + opt_fF(s, r, e) - p;
        }
        return 0;
    }
    if (!d) return 0;
    uint64_t x = match_exp(s, p + d, e, 'e');
    if (x) return d + x + opt_fF(s, p + d + x, e);
    if (p + d < e && (s[p + d] | 0x20u) == 'f') return d + 1;
    return 0;
}

template <class S>
__device__ __forceinline__ uint64_t run_ul(S s, uint64_t q, uint64_t e) {
    uint64_t r = q;
    while (r < e) {
        uint32_t c = s[r] | 0x20u;
        if (c != 'u' && c != 'l') break;
        r++;
    }
    return r - q;
}

struct Match {
    uint32_t kind;  // K_NONE = no token (whitespace, comment, skipped byte)
    uint32_t nl;    // newlines the reference adds to `line`
    uint64_t len;
};

template <class S>
__device__ Match lex_one(S s, uint64_t p, uint64_t e, const KwEntry *kw) {
    uint32_t c = s[p];
    uint32_t c1 = p + 1 < e ? s[p + 1] : 0x100u;
    uint32_t c2 = p + 2 < e ? s[p + 2] : 0x100u;
    if (c == '/' && c1 == '/') {
        uint64_t q = p + 2;
        while (q < e && s[q] != '\n') q++;
        return {K_NONE, 0, q - p};
    }
    if (c == '/' && c1 == '*') {
        uint64_t q = p + 2;
        uint32_t nl = 0;
        while (q + 1 < e) {
            uint32_t x = s[q];
            if (x == '*' && s[q + 1] == '/') return {K_NONE, nl, q + 2 - p};
            nl += x == '\n';
            q++;
        }
        // unterminated: the regex alternative fails, '/' is read as an operator
    }
    if (c == '"') {
        uint64_t q = p + 1;
        while (q < e) {
            uint32_t x = s[q];
            if (x == '"') return {K_STRING, 0, q + 1 - p};
            if (x == '\\') {
                if (q + 1 >= e) break;
                q += 2;
            } else {
                q++;
            }
        }
        return {K_NONE, 0, 1};  // unterminated: the quote matches nothing
    }
    if (c == '\'') {
        if (c1 != 0x100u && c1 != '\'' && c1 != '\\' && c2 == '\'') return {K_CHAR, 0, 3};
        if (c1 == '\\' && p + 3 < e && s[p + 3] == '\'') return {K_CHAR, 0, 4};
        return {K_NONE, 0, 1};
    }
    if (is_dig(c) || c == '.') {
        uint64_t L = match_hexfloat(s, p, e);
        if (L) return {K_FLOAT | HEXFLOAT, 0, L};
        L = match_float(s, p, e);
        if (L) return {K_FLOAT, 0, L};
        if (c == '0' && (c1 | 0x20u) == 'x') {
            uint64_t h = run_hex(s, p + 2, e);
            if (h) return {K_INT, 0, 2 + h + run_ul(s, p + 2 + h, e)};
        }
        if (c != '.') {
            uint64_t d = run_digits(s, p, e);
            return {K_INT, 0, d + run_ul(s, p + d, e)};
        }
        return {K_DOT, 0, 1};
    }
    if (is_id0(c)) {
        uint64_t q = p + 1;
        while (q < e && is_id(s[q])) q++;
        uint64_t L = q - p;
        uint32_t kind = K_IDENT;
        if (L >= 2 && L <= 15) {
            const KwEntry &k = kw[kw_hash(s, p, L)];
            if (k.len == L) {
                bool eq = true;
                for (uint64_t j = 0; j < L; ++j)
                    if ((uint8_t)k.w[j] != s[p + j]) { eq = false; break; }
                if (eq) kind = k.kind;
            }
        }
        return {kind, 0, L};
    }
    switch (c) {
    case '<':
        if (c1 == '<') return c2 == '=' ? Match{K_LSHIFT_EQ, 0, 3} : Match{K_LSHIFT, 0, 2};
        return c1 == '=' ? Match{K_LE, 0, 2} : Match{K_LT, 0, 1};
    case '>':
        if (c1 == '>') return c2 == '=' ? Match{K_RSHIFT_EQ, 0, 3} : Match{K_RSHIFT, 0, 2};
        return c1 == '=' ? Match{K_GE, 0, 2} : Match{K_GT, 0, 1};
    case '+':
        if (c1 == '+') return {K_PLUSPLUS, 0, 2};
        return c1 == '=' ? Match{K_PLUS_EQ, 0, 2} : Match{K_PLUS, 0, 1};
    case '-':
        if (c1 == '-') return {K_MINUSMINUS, 0, 2};
        if (c1 == '=') return {K_MINUS_EQ, 0, 2};
        return c1 == '>' ? Match{K_ARROW, 0, 2} : Match{K_MINUS, 0, 1};
    case '*': return c1 == '=' ? Match{K_STAR_EQ, 0, 2} : Match{K_STAR, 0, 1};
    case '/': return c1 == '=' ? Match{K_SLASH_EQ, 0, 2} : Match{K_SLASH, 0, 1};
    case '%': return c1 == '=' ? Match{K_PERCENT_EQ, 0, 2} : Match{K_PERCENT, 0, 1};
    case '&':
        if (c1 == '=') return {K_AMP_EQ, 0, 2};
        return c1 == '&' ? Match{K_AND, 0, 2} : Match{K_AMP, 0, 1};
    case '|':
        if (c1 == '=') return {K_PIPE_EQ, 0, 2};
        return c1 == '|' ? Match{K_OR, 0, 2} : Match{K_PIPE, 0, 1};
    case '^': return c1 == '=' ? Match{K_CARET_EQ, 0, 2} : Match{K_CARET, 0, 1};
    case '=': return c1 == '=' ? Match{K_EQ, 0, 2} : Match{K_ASSIGN, 0, 1};
    case '!': return c1 == '=' ? Match{K_NE, 0, 2} : Match{K_BANG, 0, 1};
    case '~': return {K_TILDE, 0, 1};
    case '(': return {K_LPAREN, 0, 1};
    case ')': return {K_RPAREN, 0, 1};
    case '{': return {K_LBRACE, 0, 1};
    case '}': return {K_RBRACE, 0, 1};
    case '[': return {K_LBRACKET, 0, 1};
    case ']': return {K_RBRACKET, 0, 1};
    case ';': return {K_SEMI, 0, 1};
    case ',': return {K_COMMA, 0, 1};
    case '?': return {K_QUESTION, 0, 1};
    case ':': return {K_COLON, 0, 1};
    case '\n': return {K_NONE, 1, 1};
    case ' ': case '\t': case '\r': {
        uint64_t q = p + 1;
        while (q < e) {
            uint32_t x = s[q];
            if (x != ' ' && x != '\t' && x != '\r') break;
            q++;
        }
        return {K_NONE, 0, q - p};
    }
    default:
        return {K_NONE, 0, 1};  // no alternative matches: skipped
    }
}

struct LexOut {
    uint32_t *start, *kindlen, *line;
    uint64_t cap;
    uint64_t *tu_tok_off;
    unsigned long long *errkey;
    uint32_t *unsup;
};

// Tokens of the segment [a, b) (a is a sync point), EOF tokens of every TU that
// ends in (a, b] (and, for a == 0, of the empty TUs at 0).  Returns the count.
template <bool WRITE>
__device__ uint64_t lex_segment(Src s, const uint64_t *__restrict__ tu_off, uint32_t n_tu,
                                uint64_t a, uint64_t b, uint32_t line, const KwEntry *kw,
                                uint64_t out0, const LexOut &o) {
    uint64_t n = 0;
    uint32_t k = upper_bound_u64(tu_off, n_tu, a) - 1;
    auto emit = [&](uint64_t pos, uint32_t kind, uint64_t len, uint32_t ln) {
        if (WRITE) {
            uint64_t i = out0 + n;
            if (i < o.cap) {
                o.start[i] = (uint32_t)pos;
                o.kindlen[i] = (kind << 24) | (uint32_t)(len > 0xFFFFFFu ? 0xFFFFFFu : len);
                if (o.line) o.line[i] = ln;
            }
        }
        n++;
    };
    if (a == 0) {
        for (uint32_t j = 0; j < k; ++j) {  // empty TUs at the very start
            emit(0, K_EOF, 0, 1);
            if (WRITE) o.tu_tok_off[j + 1] = out0 + n;
        }
    }
    uint64_t p = a, e = __ldg(tu_off + k + 1);
    for (;;) {
        while (p == e && e <= b) {  // TU k ends here: its EOF token is ours
            emit(e, K_EOF, 0, line);
            if (WRITE) o.tu_tok_off[k + 1] = out0 + n;
            ++k;
            line = 1;
            if (k >= n_tu) break;
            e = __ldg(tu_off + k + 1);
        }
        if (k >= n_tu || p >= b) break;
        Match m = lex_one(s, p, e, kw);
        if (m.kind != K_NONE) {
            emit(p, m.kind, m.len, line);
            if (WRITE) {
                if (m.kind & HEXFLOAT) {
                    uint32_t v = hexfloat_verdict(s, p, m.len);
                    if (v) atomicMin(o.errkey + k, (unsigned long long)((p << 8) | v));
                }
                if (m.len > 0xFFFFFFu) o.unsup[k] = 1;
            }
        }
        line += m.nl;
        p += m.len;
    }
    return n;
}

__global__ void __launch_bounds__(BLOCK)
k_lex_tokens(bool write, const uint8_t *__restrict__ src, uint64_t N,
             const uint64_t *__restrict__ tu_off, uint32_t n_tu, uint64_t n_win,
             const uint64_t *__restrict__ S, const uint32_t *__restrict__ sinfo,
             const uint64_t *__restrict__ nlcarry, uint64_t *__restrict__ counts,
             const uint64_t *__restrict__ toff, LexOut o) {
    const KwEntry *kw = g_kw;
    uint64_t w = (uint64_t)blockIdx.x * BLOCK + threadIdx.x;
    if (w >= n_win) return;
    uint64_t a = S[w], b = S[w + 1];
    if (a > N) a = N;
    if (b > N) b = N;
    uint64_t n = 0;
    if (a < b) {
        uint32_t si = sinfo[w];
        uint32_t line = (si & 0x80000000u) ? 1u
                        : 1u + (uint32_t)(nlcarry[w] & ~SEG_FLAG) + (si & 0x7FFFFFFFu);
        Src s{src};
        if (write)
            n = lex_segment<true>(s, tu_off, n_tu, a, b, line, kw, toff[w], o);
        else
            n = lex_segment<false>(s, tu_off, n_tu, a, b, line, kw, 0, o);
    }
    if (!write) counts[w] = n;
}

// ---------------------------------------------------------------------------
// token automaton (lex_tokdfa.cuh): one byte per loop iteration, the same
// instruction stream in every lane
// ---------------------------------------------------------------------------
__device__ const TokDfa g_tokdfa = make_tok_dfa();

struct DfaSmem {
    uint8_t next[NQ * NB];
    uint8_t acc[NQ];
    uint8_t cls[256];
};

__device__ __forceinline__ void load_dfa(DfaSmem &t) {
    const uint8_t *g = (const uint8_t *)&g_tokdfa;
    uint8_t *d = (uint8_t *)&t;
    static_assert(sizeof(DfaSmem) == sizeof(TokDfa), "table layout");
    for (uint32_t i = threadIdx.x; i < sizeof(TokDfa); i += blockDim.x) d[i] = g[i];
    __syncthreads();
}

// Source bytes through a 16-byte register window (one vector load per 16
// bytes; the buffer is 16-byte aligned, reads stay below N).
struct ByteWin {
    const uint8_t *__restrict__ src;
    uint64_t N;
    uint64_t base;
    uint4 w;
    __device__ __forceinline__ uint32_t at(uint64_t q) {
        uint64_t b = q & ~15ull;
        if (b != base) {
            base = b;
            if (b + 16 <= N) {
                w = __ldg(reinterpret_cast<const uint4 *>(src + b));
            } else {
                uint32_t x0 = 0, x1 = 0, x2 = 0, x3 = 0;
                for (uint32_t j = 0; j < 16 && b + j < N; ++j) {
                    uint32_t v = (uint32_t)__ldg(src + b + j) << (8 * (j & 3));
                    if (j < 4) x0 |= v;
                    else if (j < 8) x1 |= v;
                    else if (j < 12) x2 |= v;
                    else x3 |= v;
                }
                w = make_uint4(x0, x1, x2, x3);
            }
        }
        uint32_t k = (uint32_t)(q >> 2) & 3u;
        uint32_t v = k == 0 ? w.x : (k == 1 ? w.y : (k == 2 ? w.z : w.w));
        return (v >> (8u * ((uint32_t)q & 3u))) & 0xFFu;
    }
};

// Keyword table packed for register compares: the spelling as two 64-bit
// little-endian words (bytes past the length are zero).
struct KwPacked {
    uint64_t lo, hi;
    uint32_t len, kind;
};

__device__ __forceinline__ void load_kw_packed(KwPacked *t, const KwEntry *kw) {
    for (uint32_t i = threadIdx.x; i < 128; i += blockDim.x) {
        uint64_t lo = 0, hi = 0;
        for (uint32_t j = 0; j < 16; ++j) {
            uint64_t c = j < kw[i].len ? (uint8_t)kw[i].w[j] : 0;
            if (j < 8) lo |= c << (8 * j);
            else hi |= c << (8 * (j - 8));
        }
        t[i] = KwPacked{lo, hi, kw[i].len, kw[i].kind};
    }
}

__device__ __forceinline__ uint32_t byte_of(uint64_t lo, uint64_t hi, uint32_t j) {
    return (uint32_t)((j < 8 ? lo >> (8 * j) : hi >> (8 * (j - 8))) & 0xFFu);
}

// Keyword kind of an identifier of length L whose first 16 bytes are packed
// in (lo, hi), zero beyond L (K_IDENT when it is none).  Same perfect hash as
// the keyword table: (3L + 47 s[0] + 16 s[L-1] + s[min(2, L-1)]) mod 128.
__device__ __forceinline__ uint32_t keyword_kind_packed(uint64_t lo, uint64_t hi, uint32_t L,
                                                        const KwPacked *kw) {
    if (L < 2 || L > 15) return K_IDENT;
    uint32_t l = (uint32_t)L;
    uint32_t c0 = (uint32_t)(lo & 0xFFu), cl = byte_of(lo, hi, l - 1),
             c2 = byte_of(lo, hi, l > 2 ? 2 : l - 1);
    const KwPacked &k = kw[(3u * l + 47u * c0 + 16u * cl + c2) & 127u];
    return (k.len == l && k.lo == lo && k.hi == hi) ? k.kind : (uint32_t)K_IDENT;
}

// As lex_segment, with the token automaton: tokens starting in [a, b) (a is
// a sync point), EOF tokens of every TU that ends in (a, b] (and, for a == 0,
// of the empty TUs at 0).  Returns the count; WRITE also stores them.
// Every iteration reads one byte and computes both outcomes -- the automaton
// advances, or it died and the longest accepted prefix is committed -- as
// selects, so the lanes of a warp stay on one instruction stream.
template <bool WRITE>
__device__ uint64_t dfa_segment(ByteWin &bw, const uint64_t *__restrict__ tu_off, uint32_t n_tu,
                                uint64_t a, uint64_t b, uint32_t line, const KwPacked *kw,
                                const DfaSmem &T, uint64_t out0, const LexOut &o) {
    uint64_t n = 0;
    uint32_t k = upper_bound_u64(tu_off, n_tu, a) - 1;
    auto emit = [&](uint64_t pos, uint32_t kind, uint64_t len, uint32_t ln) {
        if (WRITE) {
            uint64_t i = out0 + n;
            if (i < o.cap) {
                o.start[i] = (uint32_t)pos;
                o.kindlen[i] = (kind << 24) | (uint32_t)(len > 0xFFFFFFu ? 0xFFFFFFu : len);
                if (o.line) o.line[i] = ln;
            }
        }
        n++;
    };
    if (a == 0) {
        for (uint32_t j = 0; j < k; ++j) {  // empty TUs at the very start
            emit(0, K_EOF, 0, 1);
            if (WRITE) o.tu_tok_off[j + 1] = out0 + n;
        }
    }
    // positions are 32-bit (a batch is below 4 GiB); the counting pass
    // (WRITE = false) tracks neither lines nor identifier bytes
    uint32_t e = (uint32_t)__ldg(tu_off + k + 1);
    const uint32_t b32 = (uint32_t)b;
    uint32_t tok = (uint32_t)a, q = (uint32_t)a, last = (uint32_t)a;
    uint32_t st = Q_START, lk = 0, nl = 0, nla = 0;
    uint64_t w0 = 0, w1 = 0;  // bytes of the current token, first 16 (WRITE)
    for (;;) {
        if (st == Q_START) {  // at a token boundary: TU ends and the segment end
            while (tok == e && e <= b32) {  // TU k ends here: its EOF token is ours
                emit(e, K_EOF, 0, line);
                if (WRITE) o.tu_tok_off[k + 1] = out0 + n;
                ++k;
                line = 1;
                if (k >= n_tu) break;
                e = (uint32_t)__ldg(tu_off + k + 1);
            }
            if (k >= n_tu || tok >= b32) break;
        }
        bool in_tu = q < e;
        uint32_t c = in_tu ? bw.at(q) : 0u;
        uint32_t cls = in_tu ? T.cls[c] : (uint32_t)B_EOT;
        uint32_t ns = T.next[st * NB + cls];
        uint32_t ac = T.acc[ns];
        bool adv = ns != Q_DEAD;
        // the commit this byte would cause if the automaton died here
        bool has = lk != 0;
        if (!adv && has && lk != ACC_SKIP) {
            uint32_t kind = lk;
            if (WRITE) {
                uint32_t L = last - tok;
                if (kind == K_IDENT) kind = keyword_kind_packed(w0, w1, L, kw);
                if (kind & HEXFLOAT) {
                    uint32_t v = hexfloat_verdict(Src{bw.src}, tok, L);
                    if (v) atomicMin(o.errkey + k, (unsigned long long)(((uint64_t)tok << 8) | v));
                }
                if (L > 0xFFFFFFu) o.unsup[k] = 1;
            }
            emit(tok, kind, last - tok, line);
        }
        uint32_t ntok = has ? last : tok + 1;
        uint32_t q1 = q + 1;
        bool acc_now = adv && ac != 0;
        if (WRITE) {
            line += (!adv && has && lk != K_STRING && lk != K_CHAR) ? nla : 0u;
            uint32_t j = q - tok;
            uint64_t cb = (uint64_t)c;
            w0 |= (adv && j < 8) ? cb << (8 * j) : 0ull;
            w1 |= (adv && j >= 8 && j < 16) ? cb << (8 * (j - 8)) : 0ull;
            uint32_t nl1 = nl + (c == '\n' ? 1u : 0u);
            nla = acc_now ? nl1 : (adv ? nla : 0u);
            nl = adv ? nl1 : 0u;
            w0 = adv ? w0 : 0ull;
            w1 = adv ? w1 : 0ull;
        }
        last = acc_now ? q1 : (adv ? last : ntok);
        lk = acc_now ? ac : (adv ? lk : 0u);
        st = adv ? ns : (uint32_t)Q_START;
        tok = adv ? tok : ntok;
        q = adv ? q1 : ntok;
    }
    return n;
}

__global__ void __launch_bounds__(BLOCK)
k_lex_tokens_dfa(bool write, const uint8_t *__restrict__ src, uint64_t N,
                 const uint64_t *__restrict__ tu_off, uint32_t n_tu, uint64_t n_win,
                 const uint64_t *__restrict__ S, const uint32_t *__restrict__ sinfo,
                 const uint64_t *__restrict__ nlcarry, uint64_t *__restrict__ counts,
                 const uint64_t *__restrict__ toff, LexOut o) {
    __shared__ DfaSmem T;
    __shared__ KwPacked kwp[128];
    load_kw_packed(kwp, g_kw);
    load_dfa(T);  // (its barrier also covers the keyword table)
    const KwPacked *kw = kwp;
    uint64_t w = (uint64_t)blockIdx.x * BLOCK + threadIdx.x;
    if (w >= n_win) return;
    uint64_t a = S[w], b = S[w + 1];
    if (a > N) a = N;
    if (b > N) b = N;
    uint64_t n = 0;
    if (a < b) {
        ByteWin bw{src, N, ~0ull, make_uint4(0, 0, 0, 0)};
        if (write) {  // only the writing pass needs the line at the sync point
            uint32_t si = sinfo[w];
            uint32_t line = (si & 0x80000000u) ? 1u
                            : 1u + (uint32_t)(nlcarry[w] & ~SEG_FLAG) + (si & 0x7FFFFFFFu);
            n = dfa_segment<true>(bw, tu_off, n_tu, a, b, line, kw, T, toff[w], o);
        } else {
            n = dfa_segment<false>(bw, tu_off, n_tu, a, b, 1u, kw, T, 0, o);
        }
    }
    if (!write) counts[w] = n;
}

// All TUs empty (no bytes at all): one EOF each.
__global__ void k_lex_all_empty(uint32_t n_tu, LexOut o) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_tu) {
        if (i < o.cap) {
            o.start[i] = 0;
            o.kindlen[i] = K_EOF << 24;
            if (o.line) o.line[i] = 1;
        }
        o.tu_tok_off[i + 1] = i + 1;
    }
}

__global__ void k_lex_finish(uint32_t n_tu, const unsigned long long *errkey,
                             const uint32_t *unsup, int32_t *status, uint64_t *tu_tok_off,
                             const uint64_t *total, uint64_t *n_tok) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_tu) {
        int32_t st = 0;
        if (unsup[i]) st = OCB_TU_UNSUPPORTED;
        else if (errkey[i] != ~0ull) st = (int32_t)(errkey[i] & 0xFFu);
        status[i] = st;
    }
    if (i == 0) {
        tu_tok_off[0] = 0;
        *n_tok = total ? *total : n_tu;
    }
}

__global__ void k_fill_u64(uint64_t *p, uint64_t n, uint64_t v) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) p[i] = v;
}
__global__ void k_set_u64(uint64_t *p, uint64_t v) { *p = v; }

struct ComposeOp {
    __device__ __forceinline__ uint64_t operator()(uint64_t a, uint64_t b) const {
        return map_compose(a, b);
    }
};
struct SegSumOp {
    __device__ __forceinline__ uint64_t operator()(uint64_t a, uint64_t b) const {
        if (b & SEG_FLAG) return b;
        return (a & SEG_FLAG) | ((a & ~SEG_FLAG) + b);
    }
};
struct MinOp {
    __device__ __forceinline__ uint64_t operator()(uint64_t a, uint64_t b) const {
        return a < b ? a : b;
    }
};

static inline void build_kw_table(KwEntry (&t)[128]) {
    static const struct { const char *w; uint8_t k; } KW[] = {
        {"__global__", 6}, {"__shared__", 7}, {"__device__", 8},
        {"__forceinline__", 8}, {"void", 9}, {"int", 10}, {"unsigned", 11},
        {"float", 12}, {"double", 13}, {"half", 14}, {"__half", 14},
        {"__half2", 14}, {"char", 15}, {"short", 16}, {"long", 17}, {"if", 18},
        {"else", 19}, {"for", 20}, {"while", 21}, {"return", 22}, {"struct", 23},
        {"union", 24}, {"__constant__", 27}, {"typedef", 25}, {"const", 26},
        {"volatile", 28}, {"break", 29}, {"continue", 30}, {"do", 31},
        {"switch", 32}, {"case", 33}, {"default", 34}, {"sizeof", 35},
        {"enum", 36}, {"static", 37}, {"inline", 37}, {"register", 37},
        {"extern", 37}, {"goto", 38}, {"class", 23}, {"signed", 42},
        {"bool", 39}, {"_Bool", 39}, {"true", 40}, {"false", 41},
    };
    memset(&t, 0, sizeof(t));
    for (auto &e : KW) {
        uint32_t L = (uint32_t)strlen(e.w);
        uint32_t c0 = (uint8_t)e.w[0], cl = (uint8_t)e.w[L - 1],
                 c2 = (uint8_t)e.w[L > 2 ? 2 : L - 1];
        uint32_t h = (3u * L + 47u * c0 + 16u * cl + c2) & 127u;
        memcpy(t[h].w, e.w, L);
        t[h].len = (uint8_t)L;
        t[h].kind = e.k;
    }
}

}  // namespace lex
}  // namespace ocb
