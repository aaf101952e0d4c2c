// Device-side lexer building blocks: the 8-state mode automaton used by the
// parallel scan, and the exact sequential token matcher used between sync
// points.
//
// The reference lexer (opencuda/frontend/lexer.py:168-295) is one ordered
// regex alternation run with re.finditer: at each position the FIRST
// alternative that matches wins, and a position where nothing matches is
// skipped.  Only four alternatives can span unbounded text or change how
// later bytes are read: // comments, /* */ comments, "strings" and 'c' char
// literals.  The mode automaton tracks exactly those; everything else (idents,
// numbers, operators) is resolved by the sequential matcher starting from a
// position that is provably a token boundary.
//
// Mode automaton.  A byte's class is derived from the byte and at most three
// bytes after it (or the run of backslashes before a '"'), never crossing a TU
// boundary.  With those classes 8 states suffice:
//   CODE  outside comments/strings            LC   inside // comment
//   BC    inside /* */ comment                STR  inside "string"
//   SKB   next byte is the opening '*' of /*  SK1..SK3  skip 1..3 bytes, then
//                                                        CODE
// Char literals are decided by lookahead ('x' or '\x' closed by a quote), so
// a failed literal never needs a retroactive re-read: the quote is simply
// skipped (the finditer skip) and the next byte is read in CODE.  A quote
// closes a string iff the run of backslashes right before it has even length,
// which is the pairing rule of "(?:[^"\\]|\\.)*" (the run cannot extend back
// past the opening quote).  The closing "*/" is seen at the '*' (class TERM1),
// which moves to SK1 so the '/' is consumed inside the comment.
//
// Unterminated strings and block comments: the reference's regex then fails
// and re-reads the opener as ordinary text.  The automaton stays in STR/BC to
// the end of the TU instead, which only removes sync points; the sequential
// matcher that owns the opener detects the failure and lexes the tail itself.
#pragma once
#include <stdint.h>

namespace ocb {
namespace lex {

enum : uint32_t {
    S_CODE = 0, S_LC = 1, S_BC = 2, S_STR = 3,
    S_SKB = 4, S_SK1 = 5, S_SK2 = 6, S_SK3 = 7
};
enum : uint32_t {
    C_OTHER = 0, C_NL, C_LCO, C_BCO, C_TERM1, C_Q3, C_Q4, C_QEND, C_QESC,
    C_NCLS
};

// Transition selector of one class: nibble s holds the next state from state
// s.  The nibble form is what __byte_perm takes as its selector.
constexpr uint32_t sel8(uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                        uint32_t a4, uint32_t a5, uint32_t a6, uint32_t a7) {
    return a0 | a1 << 4 | a2 << 8 | a3 << 12 | a4 << 16 | a5 << 20 |
           a6 << 24 | a7 << 28;
}
//                      CODE   LC     BC     STR    SKB   SK1    SK2    SK3
#define OCB_TSEL_INIT {                                                      \
    sel8(S_CODE, S_LC,   S_BC,  S_STR,  S_BC, S_CODE, S_SK1, S_SK2), /*OTH*/ \
    sel8(S_CODE, S_CODE, S_BC,  S_STR,  S_BC, S_CODE, S_SK1, S_SK2), /*NL */ \
    sel8(S_LC,   S_LC,   S_BC,  S_STR,  S_BC, S_CODE, S_SK1, S_SK2), /*LCO*/ \
    sel8(S_SKB,  S_LC,   S_BC,  S_STR,  S_BC, S_CODE, S_SK1, S_SK2), /*BCO*/ \
    sel8(S_CODE, S_LC,   S_SK1, S_STR,  S_BC, S_CODE, S_SK1, S_SK2), /*T1 */ \
    sel8(S_SK2,  S_LC,   S_BC,  S_STR,  S_BC, S_CODE, S_SK1, S_SK2), /*Q3 */ \
    sel8(S_SK3,  S_LC,   S_BC,  S_STR,  S_BC, S_CODE, S_SK1, S_SK2), /*Q4 */ \
    sel8(S_STR,  S_LC,   S_BC,  S_CODE, S_BC, S_CODE, S_SK1, S_SK2), /*QE */ \
    sel8(S_STR,  S_LC,   S_BC,  S_STR,  S_BC, S_CODE, S_SK1, S_SK2), /*QX */ \
}

// Class of byte c given the next three bytes (n1..n3) and how many of them
// exist inside the TU (nv).  For '"' the caller supplies the parity of the
// backslash run before it.
__device__ __forceinline__ uint32_t classify(uint32_t c, uint32_t n1, uint32_t n2,
                                             uint32_t n3, int nv, int bs_odd) {
    if (c == '\n') return C_NL;
    if (c == '/') {
        if (nv >= 1 && n1 == '/') return C_LCO;
        if (nv >= 1 && n1 == '*') return C_BCO;
        return C_OTHER;
    }
    if (c == '*') return (nv >= 1 && n1 == '/') ? C_TERM1 : C_OTHER;
    if (c == '\'') {
        if (nv >= 2 && n1 != '\'' && n1 != '\\' && n2 == '\'') return C_Q3;
        if (nv >= 3 && n1 == '\\' && n3 == '\'') return C_Q4;
        return C_OTHER;
    }
    if (c == '"') return bs_odd ? C_QESC : C_QEND;
    return C_OTHER;
}

__device__ __forceinline__ uint32_t next_state(uint32_t tsel, uint32_t st) {
    return (tsel >> (4 * st)) & 7u;
}

// Map composition for the scan: maps are 8 bytes (byte s = end state when the
// span is entered in state s).  compose(a, b) = "a then b".
__device__ __forceinline__ uint32_t bytes_to_nibbles(uint32_t x) {
    x = (x | (x >> 4)) & 0x00FF00FFu;
    x = (x | (x >> 8)) & 0x0000FFFFu;
    return x;
}
__device__ __forceinline__ uint64_t map_compose(uint64_t a, uint64_t b) {
    uint32_t blo = (uint32_t)b, bhi = (uint32_t)(b >> 32);
    uint32_t sl = bytes_to_nibbles((uint32_t)a);
    uint32_t sh = bytes_to_nibbles((uint32_t)(a >> 32));
    return ((uint64_t)__byte_perm(blo, bhi, sh) << 32) | __byte_perm(blo, bhi, sl);
}
constexpr uint64_t MAP_IDENTITY = 0x0706050403020100ull;

// ---------------------------------------------------------------------------
// Sequential matcher (one token at p, TU end e), restating the alternatives of
// lexer.py:168-229 in order.
// ---------------------------------------------------------------------------
enum : uint32_t {
    K_NONE = 0, K_INT = 1, K_FLOAT = 2, K_STRING = 3, K_CHAR = 4, K_IDENT = 5,
    K_PLUS = 43, K_MINUS, K_STAR, K_SLASH, K_PERCENT, K_AMP, K_PIPE, K_CARET,
    K_TILDE, K_BANG, K_LSHIFT, K_RSHIFT, K_EQ, K_NE, K_LT, K_LE, K_GT, K_GE,
    K_AND, K_OR, K_ASSIGN, K_PLUS_EQ, K_MINUS_EQ, K_STAR_EQ, K_SLASH_EQ,
    K_PERCENT_EQ, K_AMP_EQ, K_PIPE_EQ, K_CARET_EQ, K_LSHIFT_EQ, K_RSHIFT_EQ,
    K_LPAREN, K_RPAREN, K_LBRACE, K_RBRACE, K_LBRACKET, K_RBRACKET, K_SEMI,
    K_COMMA, K_DOT, K_ARROW, K_PLUSPLUS, K_MINUSMINUS, K_QUESTION, K_COLON,
    K_EOF
};
static_assert(K_EOF == 88, "TokKind numbering");
constexpr uint32_t HEXFLOAT = 0x80;

__device__ __forceinline__ bool is_dig(uint32_t c) { return c - '0' < 10u; }
__device__ __forceinline__ bool is_hex(uint32_t c) {
    return c - '0' < 10u || (c | 0x20u) - 'a' < 6u;
}
__device__ __forceinline__ bool is_id0(uint32_t c) {
    return (c | 0x20u) - 'a' < 26u || c == '_';
}
__device__ __forceinline__ bool is_id(uint32_t c) { return is_id0(c) || is_dig(c); }

struct Src {
    const uint8_t *__restrict__ s;
    __device__ __forceinline__ uint32_t operator[](uint64_t i) const { return __ldg(s + i); }
};

template <class S>
__device__ __forceinline__ uint64_t run_digits(S s, uint64_t q, uint64_t e) {
    uint64_t r = q;
    while (r < e && is_dig(s[r])) r++;
    return r - q;
}
template <class S>
__device__ __forceinline__ uint64_t run_hex(S s, uint64_t q, uint64_t e) {
    uint64_t r = q;
    while (r < e && is_hex(s[r])) r++;
    return r - q;
}
// [cC][+-]?[0-9]+ with c the lower-case exponent letter
template <class S>
__device__ __forceinline__ uint64_t match_exp(S s, uint64_t q, uint64_t e, uint32_t c) {
    if (q >= e || (s[q] | 0x20u) != c) return 0;
    uint64_t r = q + 1;
    if (r < e && (s[r] == '+' || s[r] == '-')) r++;
    uint64_t d = run_digits(s, r, e);
    return d ? r + d - q : 0;
}
template <class S>
__device__ __forceinline__ uint64_t opt_fF(S s, uint64_t q, uint64_t e) {
    return (q < e && (s[q] | 0x20u) == 'f') ? 1 : 0;
}
template <class S>
__device__ __forceinline__ uint64_t opt_fFlL(S s, uint64_t q, uint64_t e) {
    if (q >= e) return 0;
    uint32_t c = s[q] | 0x20u;
    return (c == 'f' || c == 'l') ? 1 : 0;
}

// Keyword perfect hash: (3*L + 47*s[0] + 16*s[L-1] + s[min(2,L-1)]) mod 128
// is collision-free over the 45 spellings of _KEYWORDS (lexer.py:120-166).
struct KwEntry { char w[16]; uint8_t len; uint8_t kind; };
template <class S>
__device__ __forceinline__ uint32_t kw_hash(S s, uint64_t p, uint64_t L) {
    uint32_t c0 = s[p], cl = s[p + L - 1], c2 = s[p + (L > 2 ? 2 : L - 1)];
    return (3u * (uint32_t)L + 47u * c0 + 16u * cl + c2) & 127u;
}

}  // namespace lex
}  // namespace ocb
