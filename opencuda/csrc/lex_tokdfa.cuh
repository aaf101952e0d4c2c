// Token automaton of the batch lexer: one deterministic automaton over byte
// classes whose maximal-munch run (longest accepted prefix, then restart)
// yields exactly the token stream of the reference's ordered regex
// alternation (opencuda/frontend/lexer.py:168-229) run with re.finditer.
//
// Why maximal munch is exact here.  At a position, finditer takes the FIRST
// alternative that matches.  For this alternation the first matching
// alternative is also the longest match over all alternatives, with two
// patterns needing care:
//   * /\*.*?\*/ is lazy: its automaton accepts at the first "*/" and has no
//     transition out of that state, so the longest accepted prefix is the
//     shortest comment, as in the regex;
//   * "(?:[^"\\]|\\.)*" and '(?:[^'\\]|\\.)' likewise end in states with no
//     way out.
// Every other alternative is a prefix-closed extension of the earlier ones
// where they overlap (hex float > hex int, float > int, <<= > << > <, ...),
// so "longest wins" picks the same one.  When the automaton dies, the token
// is the longest accepted prefix seen (backing up over bytes read past it:
// "0x1.8" without an exponent is the hex int "0x1", then ".8"); when no
// prefix was accepted, nothing matches and finditer skips one character
// (an unterminated string or char literal, '#', '@', '\\', non-ASCII bytes).
// An unterminated /* therefore yields "/" then lexes on from "*", again as
// the regex does.
//
// Accept codes: 0 = not accepting; ACC_SKIP = matched but produces no token
// (whitespace, newline, comments); otherwise the TokKind value emitted
// (HEXFLOAT or-ed in for hex-float literals).  Newlines inside a matched
// string or char literal do not advance the line (lexer.py:271-279); inside
// comments, whitespace runs and the newline token they do.
#pragma once
#include <stdint.h>
#include <initializer_list>
#include "lex_dfa.cuh"

namespace ocb {
namespace lex {

// ---- byte classes ----------------------------------------------------------
enum : uint8_t {
    B_OTHER = 0, B_WS, B_NL, B_0, B_19, B_HEXL, B_E, B_F, B_X, B_P, B_U, B_L, B_ID,
    B_DOT, B_PLUS, B_MINUS, B_STAR, B_SLASH, B_PCT, B_AMP, B_PIPE, B_CARET, B_TILDE,
    B_BANG, B_EQ, B_LT, B_GT, B_LPAR, B_RPAR, B_LBRC, B_RBRC, B_LBRK, B_RBRK, B_SEMI,
    B_COMMA, B_QUES, B_COLON, B_DQ, B_SQ, B_BSL, B_EOT,   // B_EOT: end of the TU
    NB
};

constexpr uint8_t byte_class(uint32_t c) {
    if (c == ' ' || c == '\t' || c == '\r') return B_WS;
    if (c == '\n') return B_NL;
    if (c == '0') return B_0;
    if (c >= '1' && c <= '9') return B_19;
    uint32_t l = c | 0x20u;
    if (l >= 'a' && l <= 'z') {
        if (l == 'e') return B_E;
        if (l == 'f') return B_F;
        if (l == 'x') return B_X;
        if (l == 'p') return B_P;
        if (l == 'u') return B_U;
        if (l == 'l') return B_L;
        if (l <= 'd') return B_HEXL;
        return B_ID;
    }
    switch (c) {
    case '_': return B_ID;
    case '.': return B_DOT;
    case '+': return B_PLUS;
    case '-': return B_MINUS;
    case '*': return B_STAR;
    case '/': return B_SLASH;
    case '%': return B_PCT;
    case '&': return B_AMP;
    case '|': return B_PIPE;
    case '^': return B_CARET;
    case '~': return B_TILDE;
    case '!': return B_BANG;
    case '=': return B_EQ;
    case '<': return B_LT;
    case '>': return B_GT;
    case '(': return B_LPAR;
    case ')': return B_RPAR;
    case '{': return B_LBRC;
    case '}': return B_RBRC;
    case '[': return B_LBRK;
    case ']': return B_RBRK;
    case ';': return B_SEMI;
    case ',': return B_COMMA;
    case '?': return B_QUES;
    case ':': return B_COLON;
    case '"': return B_DQ;
    case '\'': return B_SQ;
    case '\\': return B_BSL;
    default: return B_OTHER;
    }
}

// ---- states -----------------------------------------------------------------
enum : uint8_t {
    Q_DEAD = 0, Q_START,
    Q_WS, Q_NL, Q_SKIP1, Q_IDENT,
    Q_Z, Q_D, Q_DSUF, Q_ZX, Q_HEX, Q_HEXSUF, Q_HXM, Q_HXP, Q_HXPS, Q_HXE, Q_HXES,
    Q_DDOT, Q_DFRAC, Q_DE, Q_DES, Q_DEXP, Q_FSUF, Q_DOT,
    Q_SLASH, Q_LCOM, Q_BC0, Q_BCS, Q_BCEND, Q_SLASH_EQ,
    Q_STR, Q_STRESC, Q_STREND, Q_CH0, Q_CHESC, Q_CH1, Q_CHEND,
    Q_LT, Q_LSHIFT, Q_LSHIFT_EQ, Q_LE, Q_GT, Q_RSHIFT, Q_RSHIFT_EQ, Q_GE,
    Q_PLUS, Q_PLUSPLUS, Q_PLUS_EQ, Q_MINUS, Q_MINUSMINUS, Q_MINUS_EQ, Q_ARROW,
    Q_STAR, Q_STAR_EQ, Q_PCT, Q_PCT_EQ, Q_AMP, Q_AMP_EQ, Q_AND, Q_PIPE, Q_PIPE_EQ, Q_OR,
    Q_CARET, Q_CARET_EQ, Q_ASSIGN, Q_EQEQ, Q_BANG, Q_NE,
    Q_TILDE, Q_LPAR, Q_RPAR, Q_LBRC, Q_RBRC, Q_LBRK, Q_RBRK, Q_SEMI, Q_COMMA, Q_QUES,
    Q_COLON,
    NQ
};
constexpr uint8_t ACC_SKIP = 0xFF;

struct TokDfa {
    uint8_t next[NQ][NB];
    uint8_t acc[NQ];
    uint8_t cls[256];
};

constexpr bool is_hex_class(uint8_t b) {
    return b == B_0 || b == B_19 || b == B_HEXL || b == B_E || b == B_F;
}
constexpr bool is_ident_class(uint8_t b) {
    return b == B_0 || b == B_19 || b == B_HEXL || b == B_E || b == B_F || b == B_X ||
           b == B_P || b == B_U || b == B_L || b == B_ID;
}

constexpr TokDfa make_tok_dfa() {
    TokDfa d{};
    for (uint32_t c = 0; c < 256; ++c) d.cls[c] = byte_class(c);
    auto on = [&](uint8_t from, uint8_t b, uint8_t to) { d.next[from][b] = to; };
    auto acc = [&](uint8_t q, uint8_t k) { d.acc[q] = k; };
    // START
    on(Q_START, B_OTHER, Q_SKIP1);
    on(Q_START, B_BSL, Q_SKIP1);
    on(Q_START, B_WS, Q_WS);
    on(Q_START, B_NL, Q_NL);
    on(Q_START, B_0, Q_Z);
    on(Q_START, B_19, Q_D);
    for (uint8_t b : {B_HEXL, B_E, B_F, B_X, B_P, B_U, B_L, B_ID}) on(Q_START, b, Q_IDENT);
    on(Q_START, B_DOT, Q_DOT);
    on(Q_START, B_SLASH, Q_SLASH);
    on(Q_START, B_DQ, Q_STR);
    on(Q_START, B_SQ, Q_CH0);
    on(Q_START, B_LT, Q_LT);
    on(Q_START, B_GT, Q_GT);
    on(Q_START, B_PLUS, Q_PLUS);
    on(Q_START, B_MINUS, Q_MINUS);
    on(Q_START, B_STAR, Q_STAR);
    on(Q_START, B_PCT, Q_PCT);
    on(Q_START, B_AMP, Q_AMP);
    on(Q_START, B_PIPE, Q_PIPE);
    on(Q_START, B_CARET, Q_CARET);
    on(Q_START, B_EQ, Q_ASSIGN);
    on(Q_START, B_BANG, Q_BANG);
    on(Q_START, B_TILDE, Q_TILDE);
    on(Q_START, B_LPAR, Q_LPAR);
    on(Q_START, B_RPAR, Q_RPAR);
    on(Q_START, B_LBRC, Q_LBRC);
    on(Q_START, B_RBRC, Q_RBRC);
    on(Q_START, B_LBRK, Q_LBRK);
    on(Q_START, B_RBRK, Q_RBRK);
    on(Q_START, B_SEMI, Q_SEMI);
    on(Q_START, B_COMMA, Q_COMMA);
    on(Q_START, B_QUES, Q_QUES);
    on(Q_START, B_COLON, Q_COLON);
    // whitespace runs, newline, unmatched byte
    on(Q_WS, B_WS, Q_WS);
    acc(Q_WS, ACC_SKIP);
    acc(Q_NL, ACC_SKIP);
    acc(Q_SKIP1, ACC_SKIP);
    // identifiers
    for (uint8_t b = 0; b < NB; ++b)
        if (is_ident_class(b)) on(Q_IDENT, b, Q_IDENT);
    acc(Q_IDENT, K_IDENT);
    // decimal numbers: [0-9]+ [uUlL]* | floats
    for (uint8_t q : {Q_Z, Q_D}) {
        on(q, B_0, Q_D);
        on(q, B_19, Q_D);
        on(q, B_U, Q_DSUF);
        on(q, B_L, Q_DSUF);
        on(q, B_DOT, Q_DDOT);
        on(q, B_E, Q_DE);
        on(q, B_F, Q_FSUF);
        acc(q, K_INT);
    }
    on(Q_Z, B_X, Q_ZX);
    on(Q_DSUF, B_U, Q_DSUF);
    on(Q_DSUF, B_L, Q_DSUF);
    acc(Q_DSUF, K_INT);
    // hex ints and hex floats
    for (uint8_t b = 0; b < NB; ++b)
        if (is_hex_class(b)) {
            on(Q_ZX, b, Q_HEX);
            on(Q_HEX, b, Q_HEX);
            on(Q_HXM, b, Q_HXM);
        }
    on(Q_ZX, B_DOT, Q_HXM);
    on(Q_HEX, B_DOT, Q_HXM);
    on(Q_HEX, B_U, Q_HEXSUF);
    on(Q_HEX, B_L, Q_HEXSUF);
    on(Q_HEX, B_P, Q_HXP);
    acc(Q_HEX, K_INT);
    on(Q_HEXSUF, B_U, Q_HEXSUF);
    on(Q_HEXSUF, B_L, Q_HEXSUF);
    acc(Q_HEXSUF, K_INT);
    on(Q_HXM, B_P, Q_HXP);
    on(Q_HXP, B_PLUS, Q_HXPS);
    on(Q_HXP, B_MINUS, Q_HXPS);
    for (uint8_t q : {Q_HXP, Q_HXPS, Q_HXE}) {
        on(q, B_0, Q_HXE);
        on(q, B_19, Q_HXE);
    }
    on(Q_HXE, B_F, Q_HXES);
    on(Q_HXE, B_L, Q_HXES);
    acc(Q_HXE, K_FLOAT | HEXFLOAT);
    acc(Q_HXES, K_FLOAT | HEXFLOAT);
    // decimal floats
    for (uint8_t q : {Q_DDOT, Q_DFRAC}) {
        on(q, B_0, Q_DFRAC);
        on(q, B_19, Q_DFRAC);
        on(q, B_E, Q_DE);
        on(q, B_F, Q_FSUF);
        acc(q, K_FLOAT);
    }
    on(Q_DE, B_PLUS, Q_DES);
    on(Q_DE, B_MINUS, Q_DES);
    for (uint8_t q : {Q_DE, Q_DES, Q_DEXP}) {
        on(q, B_0, Q_DEXP);
        on(q, B_19, Q_DEXP);
    }
    on(Q_DEXP, B_F, Q_FSUF);
    acc(Q_DEXP, K_FLOAT);
    acc(Q_FSUF, K_FLOAT);
    // '.' and .[0-9]+
    on(Q_DOT, B_0, Q_DFRAC);
    on(Q_DOT, B_19, Q_DFRAC);
    acc(Q_DOT, K_DOT);
    // '/', comments, '/='
    on(Q_SLASH, B_SLASH, Q_LCOM);
    on(Q_SLASH, B_STAR, Q_BC0);
    on(Q_SLASH, B_EQ, Q_SLASH_EQ);
    acc(Q_SLASH, K_SLASH);
    acc(Q_SLASH_EQ, K_SLASH_EQ);
    for (uint8_t b = 0; b < NB; ++b)
        if (b != B_NL && b != B_EOT) on(Q_LCOM, b, Q_LCOM);
    acc(Q_LCOM, ACC_SKIP);
    for (uint8_t b = 0; b < NB; ++b)
        if (b != B_EOT) {
            on(Q_BC0, b, b == B_STAR ? Q_BCS : Q_BC0);
            on(Q_BCS, b, b == B_STAR ? Q_BCS : (b == B_SLASH ? Q_BCEND : Q_BC0));
        }
    acc(Q_BCEND, ACC_SKIP);
    // "string" and 'c'
    for (uint8_t b = 0; b < NB; ++b)
        if (b != B_EOT) {
            on(Q_STR, b, b == B_DQ ? Q_STREND : (b == B_BSL ? Q_STRESC : Q_STR));
            on(Q_STRESC, b, Q_STR);
            on(Q_CHESC, b, Q_CH1);
            if (b != B_SQ) on(Q_CH0, b, b == B_BSL ? Q_CHESC : Q_CH1);
        }
    acc(Q_STREND, K_STRING);
    on(Q_CH1, B_SQ, Q_CHEND);
    acc(Q_CHEND, K_CHAR);
    // operators, longest first as in the alternation
    on(Q_LT, B_LT, Q_LSHIFT);
    on(Q_LT, B_EQ, Q_LE);
    on(Q_LSHIFT, B_EQ, Q_LSHIFT_EQ);
    on(Q_GT, B_GT, Q_RSHIFT);
    on(Q_GT, B_EQ, Q_GE);
    on(Q_RSHIFT, B_EQ, Q_RSHIFT_EQ);
    on(Q_PLUS, B_PLUS, Q_PLUSPLUS);
    on(Q_PLUS, B_EQ, Q_PLUS_EQ);
    on(Q_MINUS, B_MINUS, Q_MINUSMINUS);
    on(Q_MINUS, B_EQ, Q_MINUS_EQ);
    on(Q_MINUS, B_GT, Q_ARROW);
    on(Q_STAR, B_EQ, Q_STAR_EQ);
    on(Q_PCT, B_EQ, Q_PCT_EQ);
    on(Q_AMP, B_EQ, Q_AMP_EQ);
    on(Q_AMP, B_AMP, Q_AND);
    on(Q_PIPE, B_EQ, Q_PIPE_EQ);
    on(Q_PIPE, B_PIPE, Q_OR);
    on(Q_CARET, B_EQ, Q_CARET_EQ);
    on(Q_ASSIGN, B_EQ, Q_EQEQ);
    on(Q_BANG, B_EQ, Q_NE);
    acc(Q_LT, K_LT); acc(Q_LSHIFT, K_LSHIFT); acc(Q_LSHIFT_EQ, K_LSHIFT_EQ); acc(Q_LE, K_LE);
    acc(Q_GT, K_GT); acc(Q_RSHIFT, K_RSHIFT); acc(Q_RSHIFT_EQ, K_RSHIFT_EQ); acc(Q_GE, K_GE);
    acc(Q_PLUS, K_PLUS); acc(Q_PLUSPLUS, K_PLUSPLUS); acc(Q_PLUS_EQ, K_PLUS_EQ);
    acc(Q_MINUS, K_MINUS); acc(Q_MINUSMINUS, K_MINUSMINUS); acc(Q_MINUS_EQ, K_MINUS_EQ);
    acc(Q_ARROW, K_ARROW);
    acc(Q_STAR, K_STAR); acc(Q_STAR_EQ, K_STAR_EQ);
    acc(Q_PCT, K_PERCENT); acc(Q_PCT_EQ, K_PERCENT_EQ);
    acc(Q_AMP, K_AMP); acc(Q_AMP_EQ, K_AMP_EQ); acc(Q_AND, K_AND);
    acc(Q_PIPE, K_PIPE); acc(Q_PIPE_EQ, K_PIPE_EQ); acc(Q_OR, K_OR);
    acc(Q_CARET, K_CARET); acc(Q_CARET_EQ, K_CARET_EQ);
    acc(Q_ASSIGN, K_ASSIGN); acc(Q_EQEQ, K_EQ);
    acc(Q_BANG, K_BANG); acc(Q_NE, K_NE);
    acc(Q_TILDE, K_TILDE); acc(Q_LPAR, K_LPAREN); acc(Q_RPAR, K_RPAREN);
    acc(Q_LBRC, K_LBRACE); acc(Q_RBRC, K_RBRACE); acc(Q_LBRK, K_LBRACKET);
    acc(Q_RBRK, K_RBRACKET); acc(Q_SEMI, K_SEMI); acc(Q_COMMA, K_COMMA);
    acc(Q_QUES, K_QUESTION); acc(Q_COLON, K_COLON);
    return d;
}

}  // namespace lex
}  // namespace ocb
