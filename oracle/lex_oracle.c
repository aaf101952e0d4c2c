/*
 * CPU restatement of the reference lexer -- TEST INFRASTRUCTURE ONLY.
 *
 * This is the oracle the GPU lexer is checked against, and the single-thread
 * CPU baseline for the lexer stage.  It is never linked into, loaded by or
 * called from the product library.
 *
 * It restates opencuda/frontend/lexer.py:258-295 (lex) over bytes:
 *   - _TOKEN_RE (lexer.py:168-229) is tried alternative by alternative, in
 *     the regex's order, at every position (re.finditer semantics: the first
 *     alternative that matches wins, not the longest; a position where no
 *     alternative matches is skipped by one character);
 *   - WS, comments and NEWLINE produce no token; `line` advances by the
 *     newlines inside WS/comments and by one per NEWLINE (lexer.py:270-276);
 *     newlines inside string or char literals are not counted;
 *   - identifiers map through _KEYWORDS (lexer.py:120-166);
 *   - a hex float keeps its source span here and carries flag 0x80 in the
 *     kind byte; the reference stores str(float.fromhex(span)) as the value
 *     (lexer.py:282-284), a pure function of the span;
 *   - each TU ends with an EOF token carrying the final line (lexer.py:294).
 * Token kinds are the numeric values of TokKind (lexer.py:11-109).
 *
 * Build: oracle/Makefile -> oracle/_ref/liblexoracle.so
 */
#include <stdint.h>
#include <string.h>

enum {
    K_INT = 1, K_FLOAT = 2, K_STRING = 3, K_CHAR = 4, K_IDENT = 5,
    K_PLUS = 43, K_MINUS, K_STAR, K_SLASH, K_PERCENT, K_AMP, K_PIPE, K_CARET,
    K_TILDE, K_BANG, K_LSHIFT, K_RSHIFT, K_EQ, K_NE, K_LT, K_LE, K_GT, K_GE,
    K_AND, K_OR, K_ASSIGN, K_PLUS_EQ, K_MINUS_EQ, K_STAR_EQ, K_SLASH_EQ,
    K_PERCENT_EQ, K_AMP_EQ, K_PIPE_EQ, K_CARET_EQ, K_LSHIFT_EQ, K_RSHIFT_EQ,
    K_LPAREN, K_RPAREN, K_LBRACE, K_RBRACE, K_LBRACKET, K_RBRACKET, K_SEMI,
    K_COMMA, K_DOT, K_ARROW, K_PLUSPLUS, K_MINUSMINUS, K_QUESTION, K_COLON,
    K_EOF
};

static const struct { const char *w; int k; } KW[] = {
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

static int is_dig(int c) { return c >= '0' && c <= '9'; }
static int is_hex(int c) {
    return is_dig(c) || (c >= 'a' && c <= 'f') || (c >= 'A' && c <= 'F');
}
static int is_id0(int c) {
    return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || c == '_';
}
static int is_id(int c) { return is_id0(c) || is_dig(c); }

static int kw_lookup(const uint8_t *s, uint64_t n) {
    for (unsigned i = 0; i < sizeof(KW) / sizeof(KW[0]); i++)
        if (strlen(KW[i].w) == n && memcmp(KW[i].w, s, n) == 0) return KW[i].k;
    return K_IDENT;
}

/* Each matcher returns the match length at p (0 = no match). */
static uint64_t m_digits(const uint8_t *s, uint64_t p, uint64_t e) {
    uint64_t q = p;
    while (q < e && is_dig(s[q])) q++;
    return q - p;
}
static uint64_t m_hexdigits(const uint8_t *s, uint64_t p, uint64_t e) {
    uint64_t q = p;
    while (q < e && is_hex(s[q])) q++;
    return q - p;
}
/* [pP][+-]?[0-9]+  or  [eE][+-]?[0-9]+ */
static uint64_t m_exp(const uint8_t *s, uint64_t p, uint64_t e, int c1, int c2) {
    uint64_t q = p;
    if (q >= e || (s[q] != c1 && s[q] != c2)) return 0;
    q++;
    if (q < e && (s[q] == '+' || s[q] == '-')) q++;
    uint64_t d = m_digits(s, q, e);
    if (!d) return 0;
    return q + d - p;
}
static uint64_t opt1(const uint8_t *s, uint64_t q, uint64_t e, const char *set) {
    return (q < e && s[q] && strchr(set, s[q])) ? 1 : 0;
}

/* HEX_FLOAT_LIT (lexer.py:173-174) */
static uint64_t m_hexfloat(const uint8_t *s, uint64_t p, uint64_t e) {
    if (p + 1 >= e || s[p] != '0' || (s[p + 1] != 'x' && s[p + 1] != 'X')) return 0;
    uint64_t q = p + 2;
    uint64_t h = m_hexdigits(s, q, e);
    /* alternative 1: hex* '.' hex* exp suffix? */
    if (q + h < e && s[q + h] == '.') {
        uint64_t r = q + h + 1;
        r += m_hexdigits(s, r, e);
        uint64_t x = m_exp(s, r, e, 'p', 'P');
        if (x) {
            r += x;
            r += opt1(s, r, e, "fFlL");
            return r - p;
        }
    }
    /* alternative 2: hex+ exp suffix? */
    if (h) {
        uint64_t r = q + h;
        uint64_t x = m_exp(s, r, e, 'p', 'P');
        if (x) {
            r += x;
            r += opt1(s, r, e, "fFlL");
            return r - p;
        }
    }
    return 0;
}

/* FLOAT_LIT (lexer.py:175-178), four alternatives in order */
static uint64_t m_float(const uint8_t *s, uint64_t p, uint64_t e) {
    uint64_t d = m_digits(s, p, e);
    /* a: [0-9]+ '.' [0-9]* (exp)? [fF]? */
    if (d && p + d < e && s[p + d] == '.') {
        uint64_t r = p + d + 1;
        r += m_digits(s, r, e);
        r += m_exp(s, r, e, 'e', 'E');
        r += opt1(s, r, e, "fF");
        return r - p;
    }
    /* b: [0-9]* '.' [0-9]+ (exp)? [fF]?  -- the greedy [0-9]* can only
       end right before the '.', and alternative a already took d>0 */
    if (p + d < e && s[p + d] == '.') {
        uint64_t r = p + d + 1;
        uint64_t f = m_digits(s, r, e);
        if (f) {
            r += f;
            r += m_exp(s, r, e, 'e', 'E');
            r += opt1(s, r, e, "fF");
            return r - p;
        }
    }
    /* c: [0-9]+ exp [fF]? */
    if (d) {
        uint64_t x = m_exp(s, p + d, e, 'e', 'E');
        if (x) {
            uint64_t r = p + d + x;
            r += opt1(s, r, e, "fF");
            return r - p;
        }
    }
    /* d: [0-9]+ [fF] */
    if (d && p + d < e && (s[p + d] == 'f' || s[p + d] == 'F')) return d + 1;
    return 0;
}

static uint64_t m_suffix_ul(const uint8_t *s, uint64_t q, uint64_t e) {
    uint64_t r = q;
    while (r < e && (s[r] == 'u' || s[r] == 'U' || s[r] == 'l' || s[r] == 'L')) r++;
    return r - q;
}

static const struct { const char *op; int k; } OPS[] = {
    {"<<=", K_LSHIFT_EQ}, {">>=", K_RSHIFT_EQ}, {"<<", K_LSHIFT},
    {">>", K_RSHIFT}, {"++", K_PLUSPLUS}, {"--", K_MINUSMINUS},
    {"+=", K_PLUS_EQ}, {"-=", K_MINUS_EQ}, {"*=", K_STAR_EQ},
    {"/=", K_SLASH_EQ}, {"%=", K_PERCENT_EQ}, {"&=", K_AMP_EQ},
    {"|=", K_PIPE_EQ}, {"^=", K_CARET_EQ}, {"==", K_EQ}, {"!=", K_NE},
    {"<=", K_LE}, {">=", K_GE}, {"&&", K_AND}, {"||", K_OR}, {"->", K_ARROW},
    {"+", K_PLUS}, {"-", K_MINUS}, {"*", K_STAR}, {"/", K_SLASH},
    {"%", K_PERCENT}, {"&", K_AMP}, {"|", K_PIPE}, {"^", K_CARET},
    {"~", K_TILDE}, {"!", K_BANG}, {"<", K_LT}, {">", K_GT}, {"=", K_ASSIGN},
    {"(", K_LPAREN}, {")", K_RPAREN}, {"{", K_LBRACE}, {"}", K_RBRACE},
    {"[", K_LBRACKET}, {"]", K_RBRACKET}, {";", K_SEMI}, {",", K_COMMA},
    {".", K_DOT}, {"?", K_QUESTION}, {":", K_COLON},
};

/* What float.fromhex(span.rstrip('fFlL')) does with a hex-float token
   (lexer.py:282-284): 0 = returns a float, 1 = ValueError (no hex digit on
   either side of the point), 2 = OverflowError (rounds to 2**1024 or more).
   CPython rounds the significand to 53 bits, ties to even. */
static int hexfloat_status(const uint8_t *s, uint64_t n) {
    uint64_t q = 2, i0 = q;
    while (q < n && is_hex(s[q])) q++;
    uint64_t ni = q - i0, f0 = 0, nf = 0;
    if (q < n && s[q] == '.') {
        q++;
        f0 = q;
        while (q < n && is_hex(s[q])) q++;
        nf = q - f0;
    }
    if (ni == 0 && nf == 0) return 1;
    q++; /* p or P */
    int neg = 0;
    if (q < n && (s[q] == '+' || s[q] == '-')) { neg = s[q] == '-'; q++; }
    int64_t E = 0;
    while (q < n && is_dig(s[q])) {
        if (E < 100000000) E = E * 10 + (s[q] - '0');
        q++;
    }
    if (neg) E = -E;
    /* digits of the significand, most significant first */
    int64_t lead = -1; /* index of the first nonzero digit in int+frac */
    uint64_t nd = ni + nf;
    for (uint64_t k = 0; k < nd; k++) {
        uint8_t c = k < ni ? s[i0 + k] : s[f0 + (k - ni)];
        if (c != '0') { lead = (int64_t)k; break; }
    }
    if (lead < 0) return 0;
    int v0 = 0;
    {
        uint8_t c = lead < (int64_t)ni ? s[i0 + lead] : s[f0 + (lead - (int64_t)ni)];
        v0 = c <= '9' ? c - '0' : (c | 0x20) - 'a' + 10;
    }
    int bl = v0 >= 8 ? 4 : v0 >= 4 ? 3 : v0 >= 2 ? 2 : 1;
    /* exponent of the leading digit's top bit */
    int64_t e2 = 4 * ((int64_t)ni - 1 - lead) + (bl - 1) + E;
    if (e2 < 1023) return 0;
    if (e2 > 1023) return 2;
    /* e2 == 1023: overflow iff the top 53 bits are all ones and bit 54 is
       one (a tie rounds to even = up, above half rounds up) */
    int bits = 0, need = 54;
    for (uint64_t k = (uint64_t)lead; k < nd && bits < need; k++) {
        uint8_t c = k < ni ? s[i0 + k] : s[f0 + (k - ni)];
        int v = c <= '9' ? c - '0' : (c | 0x20) - 'a' + 10;
        int nb = (k == (uint64_t)lead) ? bl : 4;
        for (int b = nb - 1; b >= 0 && bits < need; b--, bits++)
            if (!((v >> b) & 1)) return 0;
    }
    return bits >= need ? 2 : 0;
}

/* Lex one TU [b, e).  Returns the number of tokens (EOF included) or -1 if
   `cap` would be exceeded. */
static int64_t lex_tu(const uint8_t *s, uint64_t b, uint64_t e,
                      uint32_t *ts, uint32_t *tk, uint32_t *tl, uint64_t cap,
                      int32_t *status) {
    uint64_t n = 0;
    uint32_t line = 1;
    uint64_t p = b;
#define EMIT(kind, len)                                                        \
    do {                                                                       \
        if (n >= cap) return -1;                                               \
        ts[n] = (uint32_t)p;                                                   \
        tk[n] = ((uint32_t)(kind) << 24) | (uint32_t)((len) > 0xFFFFFF ? 0xFFFFFF : (len)); \
        tl[n] = line;                                                          \
        n++;                                                                   \
    } while (0)
    while (p < e) {
        int c = s[p];
        uint64_t L;
        /* COMMENT_LINE */
        if (c == '/' && p + 1 < e && s[p + 1] == '/') {
            L = 2;
            while (p + L < e && s[p + L] != '\n') L++;
            p += L;
            continue;
        }
        /* COMMENT_BLOCK: slash-star, shortest run, star-slash (DOTALL) */
        if (c == '/' && p + 1 < e && s[p + 1] == '*') {
            uint64_t q = p + 2, nl = 0;
            int found = 0;
            while (q + 1 < e) {
                if (s[q] == '*' && s[q + 1] == '/') { found = 1; break; }
                q++;
            }
            if (found) {
                for (uint64_t r = p; r < q; r++) nl += (s[r] == '\n');
                line += (uint32_t)nl;
                p = q + 2;
                continue;
            }
        }
        /* STRING_LIT: '"' ( [^"\\] | \\. )* '"' */
        if (c == '"') {
            uint64_t q = p + 1;
            int found = 0;
            while (q < e) {
                if (s[q] == '"') { found = 1; break; }
                if (s[q] == '\\') {
                    if (q + 1 >= e) break;
                    q += 2;
                } else {
                    q++;
                }
            }
            if (found) {
                EMIT(K_STRING, q + 1 - p);
                p = q + 1;
                continue;
            }
        }
        /* CHAR_LIT: "'" ( [^'\\] | \\. ) "'" */
        if (c == '\'') {
            if (p + 2 < e && s[p + 1] != '\'' && s[p + 1] != '\\' && s[p + 2] == '\'') {
                EMIT(K_CHAR, 3);
                p += 3;
                continue;
            }
            if (p + 3 < e && s[p + 1] == '\\' && s[p + 3] == '\'') {
                EMIT(K_CHAR, 4);
                p += 4;
                continue;
            }
        }
        if (is_dig(c) || c == '.') {
            if ((L = m_hexfloat(s, p, e))) {
                int hs = hexfloat_status(s + p, L);
                if (hs && !*status) *status = hs;
                EMIT(K_FLOAT | 0x80, L);
                p += L;
                continue;
            }
            if ((L = m_float(s, p, e))) { EMIT(K_FLOAT, L); p += L; continue; }
            if (c == '0' && p + 1 < e && (s[p + 1] == 'x' || s[p + 1] == 'X')) {
                uint64_t h = m_hexdigits(s, p + 2, e);
                if (h) {
                    L = 2 + h + m_suffix_ul(s, p + 2 + h, e);
                    EMIT(K_INT, L);
                    p += L;
                    continue;
                }
            }
            if (is_dig(c)) {
                uint64_t d = m_digits(s, p, e);
                L = d + m_suffix_ul(s, p + d, e);
                EMIT(K_INT, L);
                p += L;
                continue;
            }
        }
        if (is_id0(c)) {
            L = 1;
            while (p + L < e && is_id(s[p + L])) L++;
            EMIT(kw_lookup(s + p, L), L);
            p += L;
            continue;
        }
        {
            int matched = 0;
            for (unsigned i = 0; i < sizeof(OPS) / sizeof(OPS[0]); i++) {
                uint64_t ol = strlen(OPS[i].op);
                if (p + ol <= e && memcmp(OPS[i].op, s + p, ol) == 0) {
                    EMIT(OPS[i].k, ol);
                    p += ol;
                    matched = 1;
                    break;
                }
            }
            if (matched) continue;
        }
        if (c == ' ' || c == '\t' || c == '\r') { p++; continue; }
        if (c == '\n') { line++; p++; continue; }
        p++; /* no alternative matches: finditer skips one character */
    }
    EMIT(K_EOF, 0);
    return (int64_t)n;
#undef EMIT
}

/* Lex a batch of TUs.  tu_off has n_tu+1 entries (TU i is
   [tu_off[i], tu_off[i+1])).  Tokens of TU i land at
   [tu_tok_off[i], tu_tok_off[i+1]).  Returns the total token count, or -1 if
   `cap` is exceeded.  tu_status[i] is the hex-float verdict of the first
   hex float in TU i that the reference's lex() would raise on (1 =
   ValueError, 2 = OverflowError), else 0. */
int64_t oracle_lex_batch(const uint8_t *src, const uint64_t *tu_off, uint32_t n_tu,
                         uint32_t *tok_start, uint32_t *tok_kindlen,
                         uint32_t *tok_line, uint64_t *tu_tok_off, uint64_t cap,
                         int32_t *tu_status) {
    uint64_t n = 0;
    for (uint32_t i = 0; i < n_tu; i++) {
        tu_tok_off[i] = n;
        tu_status[i] = 0;
        int64_t k = lex_tu(src, tu_off[i], tu_off[i + 1], tok_start + n,
                           tok_kindlen + n, tok_line + n, cap - n, &tu_status[i]);
        if (k < 0) return -1;
        n += (uint64_t)k;
    }
    tu_tok_off[n_tu] = n;
    return (int64_t)n;
}
