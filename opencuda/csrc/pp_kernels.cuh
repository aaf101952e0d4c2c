// Batch preprocessor kernels for sm_100a (host driver in pp.cu).
//
// Restates opencuda/frontend/preprocess.py:178-367 (preprocess) and the
// include blanking of _resolve_includes (:125-175) for every TU of a batch.
// One thread owns one TU and walks it line by line, exactly as the reference
// does, in a private arena of global memory:
//
//   * include lines (`#\s*include\s+"..."` / `<...>` after lstrip) are
//     blanked before line splicing, as the CLI's _resolve_includes does when
//     no file resolves (a TU naming an existing file is resolved on the host);
//   * lines whose rstrip() ends in a backslash are spliced (:207-217);
//   * directives are recognised on strip() text with "#<spaces>" folded
//     (:219-330), with the reference's exact-match rules (`#else`, `#endif`
//     only when alone on the line; `#if` only when followed by a space);
//   * `#elif` is evaluated but can never be taken (the reference's
//     _is_active() includes the not-taken branch itself, :246-255);
//   * text lines: function-like macros first (<= 8 rounds, macros in
//     (-len(name), insertion) order, leftmost call each time, :333-354), then
//     object-like macros (<= 8 rounds, whole-word, :358-363); macro values and
//     arguments are re.sub replacement templates, so their backslash escapes
//     are processed (\n, \0oo, ...) and a bad escape raises re.error;
//   * `#if` expressions: object macros expanded, defined(X) -> 1/0, other
//     identifiers -> 0, integer suffixes stripped, then Python eval, any
//     exception -> True (:85-119).
//
// Object-like rounds are computed word by word: a replacement can neither
// split nor merge words (its neighbours are non-word characters), so within a
// round a word is replaced by the first macro of that name in the order and
// the words of the value are then exposed only to macros later in the order.
//
// What the engine does not reproduce is flagged OCB_TU_UNSUPPORTED (non-ASCII
// bytes in processed lines, `\g<..>` templates, non-word parameter names,
// #if expressions outside an integer subset, Python ints beyond 64 bits);
// arena exhaustion is OCB_TU_OVERFLOW (retried with a larger arena);
// a macro that keeps re-creating its own call is OCB_TU_TIMEOUT (the
// reference loops forever there).
#pragma once
#include <stdint.h>
#include "../../include/ocb.h"

namespace ocb {
namespace pp {

constexpr int MAX_DEPTH = 256;        // #if nesting
constexpr int MAX_EXPANSIONS = 4096;  // function-like expansions per line
constexpr uint32_t NONE = 0xFFFFFFFFu;

__device__ __forceinline__ bool pyspace(uint32_t c) {
    return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == 0x0b || c == 0x0c ||
           (c >= 0x1c && c <= 0x1f);
}
__device__ __forceinline__ bool isw(uint32_t c) {
    return (c | 0x20u) - 'a' < 26u || c - '0' < 10u || c == '_';
}
// A code point that Python's `\w` and `\s` both reject (Latin-1 signs and
// punctuation, general punctuation without the spaces, currency signs,
// arrows, mathematical operators, technical symbols, box drawing, shapes,
// dingbats without the circled digits, Braille, more arrows): in such a
// character the byte-wise scans here see what the reference's str-wise
// regexes see.
__device__ __forceinline__ bool neutral_cp(uint32_t c) {
    if (c >= 0x80 && c <= 0xA9) return c != 0x85 && c != 0xA0;
    if ((c >= 0xAB && c <= 0xB1) || c == 0xB4 || (c >= 0xB6 && c <= 0xB8) || c == 0xBB ||
        c == 0xBF || c == 0xD7 || c == 0xF7)
        return true;
    if (c >= 0x2000 && c <= 0x206F)
        return c > 0x200A && c != 0x2028 && c != 0x2029 && c != 0x202F && c != 0x205F;
    return (c >= 0x20A0 && c <= 0x20CF) || (c >= 0x2190 && c <= 0x23FF) ||
           (c >= 0x2500 && c <= 0x2775) || (c >= 0x2794 && c <= 0x2BFF);
}
// True when every non-ASCII character of the bytes is well-formed UTF-8 and
// neutral (above).
__device__ __forceinline__ bool neutral_utf8(const uint8_t *p, uint32_t n) {
    for (uint32_t i = 0; i < n;) {
        uint32_t b = p[i];
        if (b < 0x80) { ++i; continue; }
        uint32_t len = b >= 0xF0 ? 4 : b >= 0xE0 ? 3 : b >= 0xC0 ? 2 : 0;
        if (!len || b >= 0xF8 || i + len > n) return false;
        uint32_t cp = b & (0x7Fu >> len);
        for (uint32_t q = 1; q < len; ++q) {
            if ((p[i + q] & 0xC0) != 0x80) return false;
            cp = (cp << 6) | (p[i + q] & 0x3F);
        }
        if (!neutral_cp(cp)) return false;
        i += len;
    }
    return true;
}

enum : int { ST_OK = 0, ST_RE = OCB_TU_RAISES_REERROR, ST_UNSUP = OCB_TU_UNSUPPORTED,
             ST_OVF = OCB_TU_OVERFLOW, ST_TIMEOUT = OCB_TU_TIMEOUT };

// A TU's private arena: [out | work A | work B | pool], bump-allocated pool.
struct Ctx {
    const uint8_t *src;     // the TU's bytes
    uint32_t n;             // TU length
    uint8_t *out;
    uint32_t out_len, out_cap;
    uint8_t *wa, *wb;       // line work buffers
    uint32_t wcap;
    uint8_t *pool;
    uint32_t pool_used, pool_cap;
    int status;
    __device__ void set(int s) {
        if (status == ST_OK) status = s;
    }
    __device__ uint8_t *alloc(uint32_t bytes) {
        uint32_t a = (pool_used + 15u) & ~15u;
        if (a + bytes > pool_cap) {
            set(ST_OVF);
            return nullptr;
        }
        pool_used = a + bytes;
        return pool + a;
    }
};

struct Span {
    const uint8_t *p;
    uint32_t n;
};

// ---------------------------------------------------------------------------
// macro dictionaries: Python dict order (insertion seq, kept on redefinition)
// plus the reference's sort key (-len(name), seq); open-addressing by name
// ---------------------------------------------------------------------------
struct Macro {
    const uint8_t *name;
    uint32_t nlen;
    const uint8_t *val;     // obj: processed template; func: raw body
    uint32_t vlen;
    uint32_t seq;
    uint32_t np;            // func: number of params
    const Span *params;     // func: params
    uint8_t variadic, bad_template, live, pad;
};

struct Dict {
    Macro *slot;            // hash table of `cap` entries (cap power of two)
    uint32_t cap, count, next_seq;
    Macro **order;          // live entries in sort order (rebuilt when dirty)
    uint32_t order_n, order_cap, dirty;
};

__device__ __forceinline__ uint32_t hash_name(const uint8_t *p, uint32_t n) {
    uint32_t h = 2166136261u;
    for (uint32_t i = 0; i < n; ++i) h = (h ^ p[i]) * 16777619u;
    return h;
}
__device__ __forceinline__ bool same(const uint8_t *a, uint32_t an, const uint8_t *b, uint32_t bn) {
    if (an != bn) return false;
    for (uint32_t i = 0; i < an; ++i)
        if (a[i] != b[i]) return false;
    return true;
}
// key order: true if x comes strictly before y in sorted(-len, seq) order
__device__ __forceinline__ bool before(const Macro &x, const Macro &y) {
    return x.nlen > y.nlen || (x.nlen == y.nlen && x.seq < y.seq);
}

__device__ Macro *dict_find(Dict &d, const uint8_t *p, uint32_t n) {
    if (!d.slot) return nullptr;
    uint32_t h = hash_name(p, n) & (d.cap - 1);
    for (uint32_t i = 0; i < d.cap; ++i) {
        Macro &m = d.slot[(h + i) & (d.cap - 1)];
        if (!m.name) return nullptr;                       // never-used slot
        if (m.live && same(m.name, m.nlen, p, n)) return &m;
    }
    return nullptr;
}

// Insert or overwrite (keeping the dict position of an existing key).
__device__ Macro *dict_put(Ctx &c, Dict &d, const uint8_t *p, uint32_t n) {
    if (!d.slot) {
        d.cap = 64;
        d.slot = (Macro *)c.alloc(sizeof(Macro) * d.cap);
        if (!d.slot) return nullptr;
        for (uint32_t i = 0; i < d.cap; ++i) d.slot[i] = Macro{};
    }
    Macro *m = dict_find(d, p, n);
    if (m) return m;
    if (2 * (d.count + 1) > d.cap) {  // grow (tombstones are dropped)
        Macro *old = d.slot;
        uint32_t oc = d.cap;
        d.cap *= 2;
        d.slot = (Macro *)c.alloc(sizeof(Macro) * d.cap);
        if (!d.slot) return nullptr;
        for (uint32_t i = 0; i < d.cap; ++i) d.slot[i] = Macro{};
        d.count = 0;
        d.dirty = 1;
        for (uint32_t i = 0; i < oc; ++i)
            if (old[i].name && old[i].live) {
                uint32_t h = hash_name(old[i].name, old[i].nlen) & (d.cap - 1);
                while (d.slot[h].name) h = (h + 1) & (d.cap - 1);
                d.slot[h] = old[i];
                d.count++;
            }
    }
    uint32_t h = hash_name(p, n) & (d.cap - 1);
    while (d.slot[h].name && d.slot[h].live) h = (h + 1) & (d.cap - 1);
    Macro &s = d.slot[h];
    if (!s.name) d.count++;
    s = Macro{};
    s.name = p;
    s.nlen = n;
    s.seq = d.next_seq++;
    s.live = 1;
    d.dirty = 1;
    return &s;
}

__device__ void dict_del(Dict &d, const uint8_t *p, uint32_t n) {
    Macro *m = dict_find(d, p, n);
    if (m) {
        m->live = 0;  // tombstone: name kept so probing continues
        d.dirty = 1;
    }
}

// Live macros in sorted(-len, seq) order, rebuilt only after a change.
__device__ uint32_t dict_sorted(Ctx &c, Dict &d, Macro **&order) {
    order = nullptr;
    if (!d.slot) return 0;
    if (d.dirty || !d.order) {
        if (d.order_cap < d.cap) {
            d.order = (Macro **)c.alloc(sizeof(Macro *) * d.cap);
            if (!d.order) return 0;
            d.order_cap = d.cap;
        }
        uint32_t k = 0;
        for (uint32_t i = 0; i < d.cap; ++i)
            if (d.slot[i].name && d.slot[i].live) {
                Macro *m = &d.slot[i];
                uint32_t j = k++;
                while (j > 0 && before(*m, *d.order[j - 1])) {
                    d.order[j] = d.order[j - 1];
                    --j;
                }
                d.order[j] = m;
            }
        d.order_n = k;
        d.dirty = 0;
    }
    order = d.order;
    return d.order_n;
}

// ---------------------------------------------------------------------------
// re.sub replacement templates (sre_parse.parse_template rules for a pattern
// without groups): \a \b \f \n \r \t \v, \\, \0 + up to two octal digits,
// three octal digits; any other ASCII letter, a lone trailing backslash or a
// group reference is re.error; \g<...> is left unsupported; a backslash
// before any other character is kept with it.
// ---------------------------------------------------------------------------
__device__ int template_expand(const uint8_t *s, uint32_t n, uint8_t *dst, uint32_t cap,
                               uint32_t &out) {
    uint32_t o = 0;
    for (uint32_t i = 0; i < n; ++i) {
        uint32_t c = s[i];
        uint32_t emit1 = 0x100, emit2 = 0x100;
        if (c != '\\') {
            emit1 = c;
        } else {
            if (i + 1 >= n) return ST_RE;  // bad escape (end of pattern)
            uint32_t d = s[++i];
            switch (d) {
            case 'a': emit1 = 7; break;
            case 'b': emit1 = 8; break;
            case 'f': emit1 = 12; break;
            case 'n': emit1 = 10; break;
            case 'r': emit1 = 13; break;
            case 't': emit1 = 9; break;
            case 'v': emit1 = 11; break;
            case '\\': emit1 = '\\'; break;
            case 'g': return ST_UNSUP;
            default:
                if (d == '0') {
                    uint32_t v = 0, k = 0;
                    while (k < 2 && i + 1 < n && s[i + 1] - '0' < 8u) {
                        v = v * 8 + (s[++i] - '0');
                        ++k;
                    }
                    emit1 = v;
                } else if (d - '1' < 9u) {
                    if (d - '0' < 8u && i + 2 < n && s[i + 1] - '0' < 8u && s[i + 2] - '0' < 8u) {
                        uint32_t v = (d - '0') * 64 + (s[i + 1] - '0') * 8 + (s[i + 2] - '0');
                        if (v > 0377) return ST_RE;
                        i += 2;
                        emit1 = v;
                    } else {
                        return ST_RE;  // invalid group reference
                    }
                } else if ((d | 0x20u) - 'a' < 26u) {
                    return ST_RE;      // bad escape \<letter>
                } else {
                    emit1 = '\\';
                    emit2 = d;
                }
            }
        }
        if (emit1 >= 0x80 && emit1 < 0x100) return ST_UNSUP;  // a code point, not a byte
        if (o + 2 > cap) return ST_OVF;
        dst[o++] = (uint8_t)emit1;
        if (emit2 != 0x100) dst[o++] = (uint8_t)emit2;
    }
    out = o;
    return ST_OK;
}

// ---------------------------------------------------------------------------
// line buffers
// ---------------------------------------------------------------------------
struct LBuf {
    uint8_t *p;
    uint32_t n, cap;
    __device__ bool put(Ctx &c, uint32_t ch) {
        if (n >= cap) {
            c.set(ST_OVF);
            return false;
        }
        p[n++] = (uint8_t)ch;
        return true;
    }
    __device__ bool append(Ctx &c, const uint8_t *s, uint32_t k) {
        if (n + k > cap) {
            c.set(ST_OVF);
            return false;
        }
        for (uint32_t i = 0; i < k; ++i) p[n + i] = s[i];
        n += k;
        return true;
    }
};

// Object-like expansion of `in` into `out`, one round (see header comment).
struct Frame {
    const uint8_t *p;
    uint32_t n, i;
    const Macro *m;  // macro whose value this is (null: the line itself)
};

__device__ void obj_round(Ctx &c, Dict &obj, const uint8_t *in, uint32_t inn, LBuf &out,
                          Frame *stack) {
    int sp = 0;
    stack[0] = Frame{in, inn, 0, nullptr};
    while (sp >= 0) {
        Frame &f = stack[sp];
        if (f.i >= f.n) {
            --sp;
            continue;
        }
        uint32_t ch = f.p[f.i];
        if (!isw(ch)) {
            if (!out.put(c, ch)) return;
            f.i++;
            continue;
        }
        uint32_t j = f.i;
        while (j < f.n && isw(f.p[j])) ++j;
        const uint8_t *w = f.p + f.i;
        uint32_t wn = j - f.i;
        f.i = j;
        const Macro *m = dict_find(obj, w, wn);
        if (m && (!f.m || before(*f.m, *m))) {
            if (sp + 1 >= MAX_DEPTH) {
                c.set(ST_UNSUP);
                return;
            }
            stack[++sp] = Frame{m->val, m->vlen, 0, m};
        } else {
            if (!out.append(c, w, wn)) return;
        }
    }
}

__device__ bool bytes_equal(const uint8_t *a, uint32_t an, const uint8_t *b, uint32_t bn) {
    return same(a, an, b, bn);
}

// Whole-word replacement of `name` by `rep` (already template-processed) in
// [s, s+n) -> out.  Used for parameter substitution in macro bodies, which
// the reference does one parameter at a time over the evolving text.
__device__ void replace_word(Ctx &c, const uint8_t *s, uint32_t n, const uint8_t *name,
                             uint32_t nl, const uint8_t *rep, uint32_t rl, LBuf &out) {
    uint32_t i = 0;
    while (i < n) {
        if (isw(s[i])) {
            uint32_t j = i;
            while (j < n && isw(s[j])) ++j;
            if (same(s + i, j - i, name, nl)) {
                if (!out.append(c, rep, rl)) return;
            } else {
                if (!out.append(c, s + i, j - i)) return;
            }
            i = j;
        } else {
            if (!out.put(c, s[i])) return;
            ++i;
        }
    }
}

// re.sub(r'\s*##\s*', '', s)
__device__ void strip_paste(Ctx &c, const uint8_t *s, uint32_t n, LBuf &out) {
    uint32_t i = 0;
    while (i < n) {
        // a run of whitespace followed by ## is removed with the ## and the
        // whitespace after it
        uint32_t j = i;
        while (j < n && pyspace(s[j])) ++j;
        if (j + 1 < n && s[j] == '#' && s[j + 1] == '#') {
            j += 2;
            while (j < n && pyspace(s[j])) ++j;
            i = j;
            continue;
        }
        if (!out.put(c, s[i])) return;
        ++i;
    }
}

// ---------------------------------------------------------------------------
// function-like expansion (preprocess.py:333-354, _find_macro_call_args :51,
// _expand_func_macro :24)
// ---------------------------------------------------------------------------
// Leftmost match of \bNAME\s*\( at or after `from`; returns the match start
// and the position of '(' (NONE if none).
__device__ uint32_t find_call(const uint8_t *s, uint32_t n, const uint8_t *name, uint32_t nl,
                              uint32_t from, uint32_t &paren) {
    for (uint32_t p = from; p + nl <= n; ++p) {
        if (s[p] != name[0]) continue;
        if (p > 0 && isw(s[p - 1])) continue;
        bool eq = true;
        for (uint32_t k = 1; k < nl; ++k)
            if (s[p + k] != name[k]) { eq = false; break; }
        if (!eq) continue;
        uint32_t q = p + nl;
        while (q < n && pyspace(s[q])) ++q;
        if (q < n && s[q] == '(') {
            paren = q;
            return p;
        }
    }
    return NONE;
}

// Arguments of the call whose '(' is at `open`: stripped spans; returns the
// position after the closing ')' or NONE if unbalanced.
__device__ uint32_t call_args(const uint8_t *s, uint32_t n, uint32_t open, Span *args,
                              uint32_t max_args, uint32_t &nargs, bool &too_many) {
    int depth = 0;
    nargs = 0;
    too_many = false;
    uint32_t a0 = open + 1;
    auto push = [&](uint32_t a, uint32_t b) {
        while (a < b && pyspace(s[a])) ++a;
        while (b > a && pyspace(s[b - 1])) --b;
        if (nargs < max_args) args[nargs] = Span{s + a, b - a};
        else too_many = true;
        nargs++;
    };
    for (uint32_t i = open; i < n; ++i) {
        uint32_t ch = s[i];
        if (ch == '(') {
            depth++;
        } else if (ch == ')') {
            depth--;
            if (depth == 0) {
                push(a0, i);
                return i + 1;
            }
        } else if (ch == ',' && depth == 1) {
            push(a0, i);
            a0 = i + 1;
        }
    }
    return NONE;
}

constexpr uint32_t MAX_ARGS = 64;

// Expanded body of macro m for the given args into out.
__device__ void expand_func(Ctx &c, const Macro &m, const Span *args, uint32_t nargs,
                            LBuf &out, LBuf &t1, LBuf &t2, uint8_t *tmpl, uint32_t tcap) {
    // t1 <- body
    t1.n = 0;
    if (!t1.append(c, m.val, m.vlen)) return;
    uint32_t named = m.variadic ? m.np - 1 : m.np;
    uint32_t k = named < nargs ? named : nargs;
    for (uint32_t i = 0; i < k; ++i) {
        uint32_t rl = 0;
        int st = template_expand(args[i].p, args[i].n, tmpl, tcap, rl);
        if (st) { c.set(st); return; }
        t2.n = 0;
        replace_word(c, t1.p, t1.n, m.params[i].p, m.params[i].n, tmpl, rl, t2);
        if (c.status) return;
        LBuf x = t1; t1 = t2; t2 = x;
    }
    if (m.variadic) {
        // va = ', '.join(args[named:])
        uint32_t vl = 0;
        LBuf va{tmpl, 0, tcap};
        for (uint32_t i = named; i < nargs; ++i) {
            if (i > named && (!va.put(c, ',') || !va.put(c, ' '))) return;
            if (!va.append(c, args[i].p, args[i].n)) return;
        }
        // the joined text is itself a template
        uint8_t *vt = tmpl + va.n;
        int st = template_expand(va.p, va.n, vt, tcap - va.n, vl);
        if (st) { c.set(st); return; }
        t2.n = 0;
        static const uint8_t VA[] = {'_', '_', 'V', 'A', '_', 'A', 'R', 'G', 'S', '_', '_'};
        replace_word(c, t1.p, t1.n, VA, 11, vt, vl, t2);
        if (c.status) return;
        LBuf x = t1; t1 = t2; t2 = x;
    }
    out.n = 0;
    strip_paste(c, t1.p, t1.n, out);
}

// ---------------------------------------------------------------------------
// #if evaluation: Python eval of an integer expression (preprocess.py:114-119)
// The reference compiles first, so any syntax error -> True; at run time any
// exception -> True.  Supported: int literals (dec/hex/oct/bin, underscores),
// unary + - ~, ** * // % + - << >> & ^ | and chained comparisons.  Floats,
// strings, tuples, '/', '@' and ints beyond 64 bits are reported unsupported.
// ---------------------------------------------------------------------------
enum : int { EV_OK = 0, EV_EXC = 1, EV_SYNTAX = 2, EV_UNSUP = 3 };

// 64-bit signed arithmetic with overflow detection (true = overflow)
__device__ __forceinline__ bool add_ovf(int64_t a, int64_t b, int64_t *r) {
    uint64_t u = (uint64_t)a + (uint64_t)b;
    *r = (int64_t)u;
    return ((a >= 0) == (b >= 0)) && ((*r >= 0) != (a >= 0));
}
__device__ __forceinline__ bool sub_ovf(int64_t a, int64_t b, int64_t *r) {
    uint64_t u = (uint64_t)a - (uint64_t)b;
    *r = (int64_t)u;
    return ((a >= 0) != (b >= 0)) && ((*r >= 0) != (a >= 0));
}
__device__ __forceinline__ bool mul_ovf(int64_t a, int64_t b, int64_t *r) {
    if (a == 0 || b == 0) { *r = 0; return false; }
    if ((a == -1 && b == INT64_MIN) || (b == -1 && a == INT64_MIN)) return true;
    int64_t p = (int64_t)((uint64_t)a * (uint64_t)b);
    if (p / b != a) return true;
    *r = p;
    return false;
}

// Operators of the supported subset.  Precedence as in Python, low -> high:
// comparisons < | < ^ < & < shifts < + - < * // % < unary + - ~ < **.
enum : uint8_t {
    OP_NONE = 0, OP_LT, OP_LE, OP_GT, OP_GE, OP_EQ, OP_NE,    // comparisons
    OP_OR, OP_XOR, OP_AND, OP_SHL, OP_SHR, OP_ADD, OP_SUB,
    OP_MUL, OP_FLOORDIV, OP_MOD, OP_DIV, OP_POW,
    OP_NEG, OP_POS, OP_INV, OP_LPAREN,
    RPN_NUM, RPN_BADNUM                                      // operand items
};
__device__ __forceinline__ int prec(uint8_t op) {
    if (op <= OP_NE) return 1;
    switch (op) {
    case OP_OR: return 2;
    case OP_XOR: return 3;
    case OP_AND: return 4;
    case OP_SHL: case OP_SHR: return 5;
    case OP_ADD: case OP_SUB: return 6;
    case OP_MUL: case OP_FLOORDIV: case OP_MOD: case OP_DIV: return 7;
    case OP_NEG: case OP_POS: case OP_INV: return 8;
    case OP_POW: return 9;
    default: return 0;
    }
}

struct RpnItem {
    uint8_t op;       // operator, or RPN_NUM / RPN_BADNUM
    uint8_t chain;    // comparison: 0 first link, 1 continuation
    int64_t v;
};

// Values during evaluation.  kind: EV_OK, EV_EXC (the operation raised) or
// EV_UNSUP; errors are carried as values so that an operand skipped by a
// comparison chain's short-circuit raises nothing, as in Python.
struct EVal {
    int64_t v;
    uint8_t kind;
    uint8_t in_chain;  // a comparison chain value: v = result so far
    int64_t last;      // the chain's last operand
};

// Tokenize + shunting-yard into `out`; returns EV_OK, EV_SYNTAX or EV_UNSUP.
__device__ int to_rpn(const uint8_t *s, uint32_t n, RpnItem *out, uint32_t &no, uint8_t *ops,
                      uint8_t *opchain, uint32_t cap) {
    uint32_t nops = 0, i = 0;
    no = 0;
    bool want_operand = true, started = false, later_line = false;
    int depth = 0;
    auto emit = [&](uint8_t op, uint8_t chain, int64_t v) { out[no++] = RpnItem{op, chain, v}; };
    while (true) {
        // Python's tokenizer: spaces, tabs and form feeds separate tokens; a
        // newline inside parentheses is whitespace, blank lines before the
        // expression are skipped (an indented first line is an error), and a
        // newline after a complete expression must end the input
        uint32_t ws0 = i;
        while (i < n && (s[i] == ' ' || s[i] == '\t' || s[i] == 0x0c)) ++i;
        bool indented = i > ws0;
        if (i < n && s[i] == '#')
            while (i < n && s[i] != '\n' && s[i] != '\r') ++i;  // comment
        if (i >= n) break;
        if (s[i] == '\n' || s[i] == '\r') {
            if (depth > 0) { ++i; continue; }
            if (!started) { ++i; later_line = true; continue; }
            if (want_operand) return EV_SYNTAX;
            for (; i < n; ++i) {
                uint32_t ch = s[i];
                if (ch == '#') {
                    while (i < n && s[i] != '\n' && s[i] != '\r') ++i;
                    if (i >= n) break;
                    continue;
                }
                if (ch != ' ' && ch != '\t' && ch != 0x0c && ch != '\n' && ch != '\r')
                    return EV_SYNTAX;
            }
            {   // a last line of spaces or tabs only (no newline after it) is an
                // IndentationError in eval
                uint32_t k = n;
                bool blank_indent = false;
                while (k > 0 && s[k - 1] != '\n' && s[k - 1] != '\r') {
                    uint32_t ch = s[k - 1];
                    if (ch == ' ' || ch == '\t') blank_indent = true;
                    else if (ch != 0x0c) { blank_indent = false; break; }
                    --k;
                }
                if (blank_indent) return EV_SYNTAX;
            }
            break;
        }
        if (!started && later_line && indented) return EV_SYNTAX;  // IndentationError
        started = true;
        if (s[i] < 0x20 || s[i] == 0x7f) return EV_SYNTAX;  // non-printable character
        if (no + 2 >= cap || nops + 2 >= cap) return EV_UNSUP;
        uint32_t c = s[i], c1 = i + 1 < n ? s[i + 1] : 0;
        if (c - '0' < 10u) {
            if (!want_operand) return EV_SYNTAX;
            uint32_t a = i;
            while (i < n && isw(s[i])) ++i;
            if (i < n && s[i] == '.') return EV_UNSUP;
            uint32_t L = i - a, k = 0, base = 10;
            const uint8_t *p = s + a;
            if (L >= 2 && p[0] == '0' && ((p[1] | 0x20u) == 'x' || (p[1] | 0x20u) == 'o' ||
                                         (p[1] | 0x20u) == 'b')) {
                base = (p[1] | 0x20u) == 'x' ? 16 : (p[1] | 0x20u) == 'o' ? 8 : 2;
                k = 2;
                if (k >= L) return EV_SYNTAX;
            } else if (p[0] == '0') {
                for (uint32_t j = 0; j < L; ++j)
                    if (p[j] != '0' && p[j] != '_') return EV_SYNTAX;
            }
            uint64_t v = 0;
            bool need_digit = true, big = false;
            for (; k < L; ++k) {
                uint32_t ch = p[k];
                if (ch == '_') {
                    if (need_digit) return EV_SYNTAX;
                    need_digit = true;
                    continue;
                }
                if (base == 10 && ((ch | 0x20u) == 'e' || (ch | 0x20u) == 'j')) return EV_UNSUP;
                uint32_t d = ch - '0' < 10u ? ch - '0'
                           : (ch | 0x20u) - 'a' < 6u ? (ch | 0x20u) - 'a' + 10 : 99;
                if (d >= base) return EV_SYNTAX;
                if (v > (0x7FFFFFFFFFFFFFFFull - d) / base) big = true;
                else v = v * base + d;
                need_digit = false;
            }
            if (need_digit) return EV_SYNTAX;
            emit(big ? RPN_BADNUM : RPN_NUM, 0, (int64_t)v);
            want_operand = false;
            continue;
        }
        if (c == '(') {
            if (!want_operand) return EV_UNSUP;  // a call: int object is not callable (TypeError) or worse
            ops[nops] = OP_LPAREN;
            opchain[nops++] = 0;
            ++depth;
            ++i;
            continue;
        }
        if (c == ')') {
            // "()" is the empty tuple
            if (want_operand) return nops && ops[nops - 1] == OP_LPAREN ? EV_UNSUP : EV_SYNTAX;
            while (nops && ops[nops - 1] != OP_LPAREN) { --nops; emit(ops[nops], opchain[nops], 0); }
            if (!nops) return EV_SYNTAX;
            --nops;
            --depth;
            ++i;
            continue;
        }
        uint8_t op = OP_NONE;
        uint32_t len = 1;
        if (want_operand) {
            if (c == '-') op = OP_NEG;
            else if (c == '+') op = OP_POS;
            else if (c == '~') op = OP_INV;
            else if (c == '.' || c == '"' || c == '\'' || c == '[' || c == '{' || c == '@' ||
                     c == '\\' || c == ',' || c >= 0x80) return EV_UNSUP;
            else return EV_SYNTAX;
            ops[nops] = op;  // prefix operator
            opchain[nops++] = 0;
            ++i;
            continue;
        }
        if (c == '*' && c1 == '*') { op = OP_POW; len = 2; }
        else if (c == '/' && c1 == '/') { op = OP_FLOORDIV; len = 2; }
        else if (c == '<' && c1 == '<') { op = OP_SHL; len = 2; }
        else if (c == '>' && c1 == '>') { op = OP_SHR; len = 2; }
        else if (c == '<' && c1 == '=') { op = OP_LE; len = 2; }
        else if (c == '>' && c1 == '=') { op = OP_GE; len = 2; }
        else if (c == '=' && c1 == '=') { op = OP_EQ; len = 2; }
        else if (c == '!' && c1 == '=') { op = OP_NE; len = 2; }
        else if (c == '<') op = OP_LT;
        else if (c == '>') op = OP_GT;
        else if (c == '|') op = OP_OR;
        else if (c == '^') op = OP_XOR;
        else if (c == '&') op = OP_AND;
        else if (c == '+') op = OP_ADD;
        else if (c == '-') op = OP_SUB;
        else if (c == '*') op = OP_MUL;
        else if (c == '%') op = OP_MOD;
        else if (c == '/') op = OP_DIV;
        else if (c == '.' || c == '"' || c == '\'' || c == '[' || c == '{' || c == '@' ||
                 c == '\\' || c == ',' || c >= 0x80) return EV_UNSUP;
        else return EV_SYNTAX;
        i += len;
        int p = prec(op);
        uint8_t chain = 0;
        if (p == 1) {
            // comparisons chain: pop everything above the chain level; a
            // comparison already on the stack is the previous link
            while (nops && ops[nops - 1] != OP_LPAREN && prec(ops[nops - 1]) > 1) {
                --nops;
                emit(ops[nops], opchain[nops], 0);
            }
            if (nops && ops[nops - 1] != OP_LPAREN && prec(ops[nops - 1]) == 1) {
                --nops;
                emit(ops[nops], opchain[nops], 0);
                chain = 1;
            }
        } else {
            // left-associative, except ** (right); prefix operators below **
            // stay on the stack when ** arrives
            while (nops && ops[nops - 1] != OP_LPAREN) {
                int q = prec(ops[nops - 1]);
                bool pop = op == OP_POW ? q > p : q >= p;
                if (!pop) break;
                --nops;
                emit(ops[nops], opchain[nops], 0);
            }
        }
        ops[nops] = op;
        opchain[nops++] = chain;
        want_operand = true;
    }
    if (want_operand) return EV_SYNTAX;
    while (nops) {
        --nops;
        if (ops[nops] == OP_LPAREN) return EV_SYNTAX;
        emit(ops[nops], opchain[nops], 0);
    }
    return EV_OK;
}

__device__ EVal ev_bin(uint8_t op, EVal a, EVal b) {
    EVal r{0, EV_OK, 0, 0};
    if (a.kind != EV_OK) return a;
    if (b.kind != EV_OK) return b;
    int64_t x = a.v, y = b.v;
    switch (op) {
    case OP_OR: r.v = x | y; break;
    case OP_XOR: r.v = x ^ y; break;
    case OP_AND: r.v = x & y; break;
    case OP_ADD: if (add_ovf(x, y, &r.v)) r.kind = EV_UNSUP; break;
    case OP_SUB: if (sub_ovf(x, y, &r.v)) r.kind = EV_UNSUP; break;
    case OP_MUL: if (mul_ovf(x, y, &r.v)) r.kind = EV_UNSUP; break;
    case OP_DIV: r.kind = EV_UNSUP; break;  // a float result
    case OP_FLOORDIV:
        if (y == 0) { r.kind = EV_EXC; break; }
        if (x == INT64_MIN && y == -1) { r.kind = EV_UNSUP; break; }
        r.v = x / y;
        if ((x % y != 0) && ((x < 0) != (y < 0))) r.v -= 1;
        break;
    case OP_MOD:
        if (y == 0) { r.kind = EV_EXC; break; }
        if (y == -1) { r.v = 0; break; }
        r.v = x % y;
        if (r.v != 0 && ((r.v < 0) != (y < 0))) r.v += y;
        break;
    case OP_SHL:
        if (y < 0) { r.kind = EV_EXC; break; }
        if (x != 0 && (y >= 63 || (x > 0 ? x > (INT64_MAX >> y) : x < (INT64_MIN >> y)))) {
            r.kind = EV_UNSUP;
            break;
        }
        r.v = x == 0 ? 0 : x * ((int64_t)1 << y);
        break;
    case OP_SHR:
        if (y < 0) { r.kind = EV_EXC; break; }
        r.v = y >= 63 ? (x < 0 ? -1 : 0) : (x >> y);
        break;
    case OP_POW: {
        if (y < 0) { r.kind = EV_UNSUP; break; }  // a float result
        int64_t acc = 1;
        for (int64_t k = 0; k < y; ++k) {
            if (mul_ovf(acc, x, &acc)) { r.kind = EV_UNSUP; break; }
            if (acc == 0 || acc == 1) break;
            if (acc == -1) { acc = ((y - k - 1) & 1) ? 1 : -1; break; }
        }
        r.v = acc;
        break;
    }
    default: r.kind = EV_UNSUP;
    }
    return r;
}

__device__ bool cmp(uint8_t op, int64_t x, int64_t y) {
    switch (op) {
    case OP_LT: return x < y;
    case OP_LE: return x <= y;
    case OP_GT: return x > y;
    case OP_GE: return x >= y;
    case OP_EQ: return x == y;
    default: return x != y;
    }
}

// A chain value used as an operand becomes its truth value.
__device__ __forceinline__ EVal settle(EVal a) {
    if (a.in_chain && a.kind == EV_OK) return EVal{a.v ? 1 : 0, EV_OK, 0, 0};
    a.in_chain = 0;
    return a;
}

// Evaluate `e` per _eval_if_expr's final step.  Returns 1/0 (true/false) or
// -1 when unsupported.  Scratch: 3 * (n + 8) items from the TU pool.
__device__ int py_eval_bool(Ctx &c, const uint8_t *e, uint32_t n) {
    uint32_t cap = n + 8;
    RpnItem *rpn = (RpnItem *)c.alloc(sizeof(RpnItem) * cap);
    uint8_t *ops = c.alloc(2 * cap);
    EVal *st = (EVal *)c.alloc(sizeof(EVal) * cap);
    if (!rpn || !ops || !st) return 1;
    uint32_t nr = 0;
    int r = to_rpn(e, n, rpn, nr, ops, ops + cap, cap);
    if (r == EV_SYNTAX) return 1;
    if (r == EV_UNSUP) return -1;
    uint32_t sp = 0;
    for (uint32_t k = 0; k < nr; ++k) {
        RpnItem it = rpn[k];
        if (it.op == RPN_NUM || it.op == RPN_BADNUM) {
            st[sp++] = EVal{it.v, (uint8_t)(it.op == RPN_NUM ? EV_OK : EV_UNSUP), 0, 0};
            continue;
        }
        if (it.op == OP_NEG || it.op == OP_POS || it.op == OP_INV) {
            EVal a = settle(st[sp - 1]);
            if (a.kind == EV_OK) {
                if (it.op == OP_NEG) {
                    if (a.v == INT64_MIN) a.kind = EV_UNSUP;
                    else a.v = -a.v;
                } else if (it.op == OP_INV) {
                    a.v = ~a.v;
                }
            }
            st[sp - 1] = a;
            continue;
        }
        EVal b = st[--sp];
        EVal a = st[--sp];
        if (prec(it.op) == 1) {
            b = settle(b);
            EVal out{0, EV_OK, 1, 0};
            if (!it.chain) {
                a = settle(a);
                if (a.kind != EV_OK) out = a;
                else if (b.kind != EV_OK) out = b;
                else out = EVal{cmp(it.op, a.v, b.v) ? 1 : 0, EV_OK, 1, b.v};
            } else {
                // a is the chain so far; a false chain skips b entirely
                if (a.kind != EV_OK) out = a;
                else if (!a.v) out = a;
                else if (b.kind != EV_OK) out = b;
                else out = EVal{cmp(it.op, a.last, b.v) ? 1 : 0, EV_OK, 1, b.v};
            }
            out.in_chain = 1;
            st[sp++] = out;
            continue;
        }
        st[sp++] = ev_bin(it.op, settle(a), settle(b));
    }
    EVal res = settle(st[0]);
    if (res.kind == EV_UNSUP) return -1;
    if (res.kind == EV_EXC) return 1;
    return res.v != 0;
}

// ---------------------------------------------------------------------------
// per-TU driver
// ---------------------------------------------------------------------------
struct TU {
    Ctx c;
    Dict obj, fn;
    uint8_t inc[MAX_DEPTH], seen[MAX_DEPTH];
    int depth;
    bool first_line;
    Frame *stack;           // object-expansion stack (MAX_DEPTH frames)
    uint8_t *tmpl;          // template scratch
    uint32_t tcap;
    LBuf t1, t2;            // body-expansion scratch

    __device__ bool active(int upto) const {
        for (int k = 0; k < upto; ++k)
            if (!inc[k]) return false;
        return true;
    }
    __device__ void emit_line(const uint8_t *p, uint32_t n) {
        if (c.status) return;
        uint32_t need = n + (first_line ? 0 : 1);
        if (c.out_len + need > c.out_cap) { c.set(ST_OVF); return; }
        if (!first_line) c.out[c.out_len++] = '\n';
        for (uint32_t i = 0; i < n; ++i) c.out[c.out_len + i] = p[i];
        c.out_len += n;
        first_line = false;
    }
    __device__ bool any_live(Dict &d) {
        Macro **o;
        return dict_sorted(c, d, o) > 0;
    }
    // re.sub over every live object macro: a bad template raises on any call
    __device__ bool obj_templates_ok(Dict &d) {
        Macro **o;
        uint32_t k = dict_sorted(c, d, o);
        for (uint32_t j = 0; j < k; ++j)
            if (o[j]->bad_template) { c.set(o[j]->bad_template == 1 ? ST_RE : ST_UNSUP); return false; }
        return true;
    }
    // Object-like rounds over [buf, n) -> result in *res (ping-pong a/b).
    __device__ void obj_expand(LBuf &a, LBuf &b, LBuf *&res) {
        res = &a;
        if (!any_live(obj)) return;
        if (!obj_templates_ok(obj)) return;
        for (int round = 0; round < 8; ++round) {
            b.n = 0;
            obj_round(c, obj, a.p, a.n, b, stack);
            if (c.status) return;
            bool eq = bytes_equal(a.p, a.n, b.p, b.n);
            LBuf x = a; a = b; b = x;
            res = &a;
            if (eq) break;
        }
    }
    // _eval_if_expr: the expression text is [p, n)
    __device__ int eval_if(const uint8_t *p, uint32_t n) {
        LBuf a{c.wb, 0, c.wcap / 2}, b{c.wb + c.wcap / 2, 0, c.wcap / 2};
        if (!a.append(c, p, n)) return 1;
        LBuf *r;
        obj_expand(a, b, r);
        if (c.status) return 1;
        LBuf cur = *r, oth = (r == &a) ? b : a;
        // defined(X) / defined X -> 1/0 (no word boundary before "defined")
        for (int pass = 0; pass < 2; ++pass) {
            oth.n = 0;
            uint32_t i = 0;
            while (i < cur.n) {
                bool m = false;
                if (i + 7 <= cur.n && same(cur.p + i, 7, (const uint8_t *)"defined", 7)) {
                    uint32_t j = i + 7, ws = j;
                    while (j < cur.n && pyspace(cur.p[j])) ++j;
                    if (pass == 0) {
                        if (j < cur.n && cur.p[j] == '(') {
                            ++j;
                            while (j < cur.n && pyspace(cur.p[j])) ++j;
                            uint32_t w0 = j;
                            while (j < cur.n && isw(cur.p[j])) ++j;
                            uint32_t w1 = j;
                            while (j < cur.n && pyspace(cur.p[j])) ++j;
                            if (w1 > w0 && j < cur.n && cur.p[j] == ')') {
                                bool d = dict_find(obj, cur.p + w0, w1 - w0) != nullptr;
                                if (!oth.put(c, d ? '1' : '0')) return 1;
                                i = j + 1;
                                m = true;
                            }
                        }
                    } else if (j > ws) {
                        uint32_t w0 = j;
                        while (j < cur.n && isw(cur.p[j])) ++j;
                        if (j > w0) {
                            bool d = dict_find(obj, cur.p + w0, j - w0) != nullptr;
                            if (!oth.put(c, d ? '1' : '0')) return 1;
                            i = j;
                            m = true;
                        }
                    }
                }
                if (!m) {
                    if (!oth.put(c, cur.p[i])) return 1;
                    ++i;
                }
            }
            LBuf x = cur; cur = oth; oth = x;
        }
        // identifiers -> 0, then (\d+)[uUlL]+ -> \1
        oth.n = 0;
        for (uint32_t i = 0; i < cur.n;) {
            uint32_t ch = cur.p[i];
            if (ch >= 0x80) { c.set(ST_UNSUP); return 1; }
            if (isw(ch)) {
                uint32_t j = i;
                while (j < cur.n && isw(cur.p[j])) ++j;
                if (!(ch - '0' < 10u)) {
                    if (!oth.put(c, '0')) return 1;
                } else if (!oth.append(c, cur.p + i, j - i)) {
                    return 1;
                }
                i = j;
            } else {
                if (!oth.put(c, ch)) return 1;
                ++i;
            }
        }
        { LBuf x = cur; cur = oth; oth = x; }
        oth.n = 0;
        for (uint32_t i = 0; i < cur.n;) {
            uint32_t ch = cur.p[i];
            if (ch - '0' < 10u) {
                uint32_t j = i;
                while (j < cur.n && cur.p[j] - '0' < 10u) ++j;
                uint32_t k = j;
                while (k < cur.n && ((cur.p[k] | 0x20u) == 'u' || (cur.p[k] | 0x20u) == 'l')) ++k;
                if (!oth.append(c, cur.p + i, j - i)) return 1;
                i = k;
            } else {
                if (!oth.put(c, ch)) return 1;
                ++i;
            }
        }
        int v = py_eval_bool(c, oth.p, oth.n);
        if (v < 0) { c.set(ST_UNSUP); return 1; }
        return v;
    }

    __device__ void define(const uint8_t *d, uint32_t n) {
        // d = normalized directive text starting with "#define"
        uint32_t i = 7;
        uint32_t ws0 = i;
        while (i < n && pyspace(d[i])) ++i;
        if (i == ws0) return;  // no \s+ : not a define form
        uint32_t nm0 = i;
        while (i < n && isw(d[i])) ++i;
        uint32_t nm1 = i;
        if (nm1 == nm0) return;
        const uint8_t *name = d + nm0;
        uint32_t nl = nm1 - nm0;
        if (i < n && d[i] == '(') {
            uint32_t j = i + 1;
            while (j < n && d[j] != ')') ++j;
            if (j < n) {  // function-like
                uint32_t p0 = i + 1, p1 = j;
                uint32_t b0 = j + 1;
                while (b0 < n && pyspace(d[b0])) ++b0;
                // body = rest.strip(), then re.sub(r'\s*//.*$', '', body)
                uint32_t b1 = n;
                while (b1 > b0 && pyspace(d[b1 - 1])) --b1;
                for (uint32_t k = b0; k + 1 < b1; ++k)
                    if (d[k] == '/' && d[k + 1] == '/') {
                        uint32_t e = k;
                        while (e > b0 && pyspace(d[e - 1])) --e;
                        b1 = e;
                        break;
                    }
                // params: split on ',', strip, drop empty
                uint32_t np = 0;
                for (uint32_t k = p0; k <= p1; ++k) np += (k == p1 || d[k] == ',');
                Span *ps = (Span *)c.alloc(sizeof(Span) * (np ? np : 1));
                uint8_t *copy = c.alloc(n);
                if (!ps || !copy) return;
                for (uint32_t k = 0; k < n; ++k) copy[k] = d[k];
                uint32_t cnt = 0, a = p0;
                bool variadic = false;
                for (uint32_t k = p0; k <= p1; ++k) {
                    if (k < p1 && d[k] != ',') continue;
                    uint32_t x = a, y = k;
                    while (x < y && pyspace(d[x])) ++x;
                    while (y > x && pyspace(d[y - 1])) --y;
                    if (y > x) ps[cnt++] = Span{copy + x, y - x};
                    a = k + 1;
                }
                for (uint32_t k = 0; k < cnt; ++k) {
                    bool dots = ps[k].n == 3 && ps[k].p[0] == '.' && ps[k].p[1] == '.' && ps[k].p[2] == '.';
                    if (dots && k == cnt - 1) { variadic = true; continue; }
                    for (uint32_t q = 0; q < ps[k].n; ++q)
                        if (!isw(ps[k].p[q])) { c.set(ST_UNSUP); return; }
                }
                Macro *m = dict_put(c, fn, copy + nm0, nl);
                if (!m) return;
                m->val = copy + b0;
                m->vlen = b1 > b0 ? b1 - b0 : 0;
                m->np = cnt;
                m->params = ps;
                m->variadic = variadic;
                return;
            }
        }
        // object-like: #define NAME\s+(.*)  or  #define NAME\s*$
        uint32_t v0 = i;
        while (v0 < n && pyspace(d[v0])) ++v0;
        if (v0 == i) {
            if (i == n) {  // bare #define NAME
                uint8_t *copy = c.alloc(nl + 1);
                if (!copy) return;
                for (uint32_t k = 0; k < nl; ++k) copy[k] = name[k];
                copy[nl] = '1';
                Macro *m = dict_put(c, obj, copy, nl);
                if (!m) return;
                m->val = copy + nl;
                m->vlen = 1;
                m->bad_template = 0;
            }
            return;  // NAME followed by a non-space: not a define form
        }
        uint32_t v1 = n;  // value = rest.strip(); cut \s*//.*$; strip again
        for (uint32_t k = v0; k + 1 < v1; ++k)
            if (d[k] == '/' && d[k + 1] == '/') { v1 = k; break; }
        while (v1 > v0 && pyspace(d[v1 - 1])) --v1;
        uint8_t *copy = c.alloc(nl + 2 * (v1 - v0) + 2);
        if (!copy) return;
        for (uint32_t k = 0; k < nl; ++k) copy[k] = name[k];
        Macro *m = dict_put(c, obj, copy, nl);
        if (!m) return;
        uint32_t out = 0;
        int st = template_expand(d + v0, v1 - v0, copy + nl, 2 * (v1 - v0) + 2, out);
        if (st == ST_OVF) { c.set(ST_OVF); return; }
        m->val = copy + nl;
        m->vlen = st ? 0 : out;
        m->bad_template = (uint8_t)(st == ST_RE ? 1 : st == ST_UNSUP ? 2 : 0);
    }

    __device__ void undef(const uint8_t *d, uint32_t n) {
        uint32_t i = 6, ws0 = i;
        while (i < n && pyspace(d[i])) ++i;
        if (i == ws0) return;
        uint32_t w0 = i;
        while (i < n && isw(d[i])) ++i;
        if (i == w0) return;
        dict_del(obj, d + w0, i - w0);
        dict_del(fn, d + w0, i - w0);
    }

    __device__ void text_line(const uint8_t *line, uint32_t n) {
        LBuf a{c.wb, 0, c.wcap / 2}, b{c.wb + c.wcap / 2, 0, c.wcap / 2};
        if (!a.append(c, line, n)) return;
        bool has_macros = any_live(fn) || any_live(obj);
        if (has_macros && !neutral_utf8(line, n)) { c.set(ST_UNSUP); return; }
        Macro **order;
        uint32_t nf = dict_sorted(c, fn, order);
        if (nf) {
            uint32_t expansions = 0;
            Span args[MAX_ARGS];
            for (int round = 0; round < 8; ++round) {
                bool changed = false;
                nf = dict_sorted(c, fn, order);
                for (uint32_t mi = 0; mi < nf; ++mi) {
                    const Macro &m = *order[mi];
                    uint32_t from = 0;
                    for (;;) {
                        uint32_t paren;
                        uint32_t p = find_call(a.p, a.n, m.name, m.nlen, from, paren);
                        if (p == NONE) break;
                        uint32_t nargs;
                        bool too_many;
                        uint32_t end = call_args(a.p, a.n, paren, args, MAX_ARGS, nargs, too_many);
                        if (end == NONE) break;
                        if (too_many) { c.set(ST_UNSUP); return; }
                        if (++expansions > MAX_EXPANSIONS) { c.set(ST_TIMEOUT); return; }
                        LBuf e{b.p, 0, b.cap};
                        expand_func(c, m, args, nargs, e, t1, t2, tmpl, tcap);
                        if (c.status) return;
                        // new line = a[0:p] + e + a[end:]   (built in b)
                        uint32_t tail = a.n - end;
                        uint32_t nn = p + e.n + tail;
                        if (nn > b.cap) { c.set(ST_OVF); return; }
                        // e already sits at b.p; move it right by p, then frame
                        for (uint32_t k = e.n; k-- > 0;) b.p[p + k] = b.p[k];
                        for (uint32_t k = 0; k < p; ++k) b.p[k] = a.p[k];
                        for (uint32_t k = 0; k < tail; ++k) b.p[p + e.n + k] = a.p[end + k];
                        b.n = nn;
                        LBuf x = a; a = b; b = x;
                        changed = true;
                        // the next match can start no earlier than the word
                        // that ends right before the spaces before p
                        uint32_t q = p;
                        while (q > 0 && pyspace(a.p[q - 1])) --q;
                        while (q > 0 && isw(a.p[q - 1])) --q;
                        from = q;
                    }
                }
                if (!changed) break;
            }
        }
        LBuf *r = &a;
        obj_expand(a, b, r);
        if (c.status) return;
        emit_line(r->p, r->n);
    }

    __device__ void joined_line(const uint8_t *line, uint32_t n) {
        if (c.status) return;
        // stripped, with "#<spaces>" folded to "#"
        uint32_t a = 0, b = n;
        while (a < b && pyspace(line[a])) ++a;
        while (b > a && pyspace(line[b - 1])) --b;
        const uint8_t *d = line + a;
        uint32_t dn = b - a;
        uint8_t *norm = nullptr;
        if (dn && d[0] == '#') {
            uint32_t k = 1;
            while (k < dn && pyspace(d[k])) ++k;
            if (k > 1) {  // build "#" + rest in the template scratch
                norm = tmpl;
                norm[0] = '#';
                for (uint32_t q = k; q < dn; ++q) norm[1 + q - k] = d[q];
                dn = dn - k + 1;
                d = norm;
            }
        }
        auto starts = [&](const char *w) {
            uint32_t k = 0;
            while (w[k]) {
                if (k >= dn || d[k] != (uint8_t)w[k]) return false;
                ++k;
            }
            return true;
        };
        auto equals = [&](const char *w) {
            uint32_t k = 0;
            while (w[k]) ++k;
            return k == dn && starts(w);
        };
        if (starts("#ifdef") || starts("#ifndef")) {
            bool is_ifdef = starts("#ifdef");
            uint32_t i = is_ifdef ? 6 : 7, ws0 = i;
            while (i < dn && pyspace(d[i])) ++i;
            uint32_t w0 = i;
            while (i < dn && isw(d[i])) ++i;
            bool defined = false;
            if (i > w0 && w0 > ws0)
                defined = dict_find(obj, d + w0, i - w0) || dict_find(fn, d + w0, i - w0);
            bool taking = (is_ifdef ? defined : !defined) && active(depth);
            if (depth >= MAX_DEPTH) { c.set(ST_UNSUP); return; }
            inc[depth] = seen[depth] = taking;
            depth++;
            emit_line(nullptr, 0);
            return;
        }
        if (starts("#if ") || equals("#if")) {
            uint32_t r0 = 3, r1 = dn;
            while (r0 < r1 && pyspace(d[r0])) ++r0;
            // the expression is evaluated even in an inactive region
            uint8_t *copy = c.alloc(r1 - r0 + 1);
            if (!copy) return;
            for (uint32_t k = r0; k < r1; ++k) copy[k - r0] = d[k];
            int v = eval_if(copy, r1 - r0);
            if (c.status == ST_UNSUP && !active(depth)) c.status = ST_OK;
            if (c.status) return;
            bool taking = v && active(depth);
            if (depth >= MAX_DEPTH) { c.set(ST_UNSUP); return; }
            inc[depth] = seen[depth] = taking;
            depth++;
            emit_line(nullptr, 0);
            return;
        }
        if (starts("#elif")) {
            if (depth) {
                if (seen[depth - 1]) {
                    inc[depth - 1] = 0;
                    seen[depth - 1] = 1;
                } else {
                    uint32_t r0 = 5, r1 = dn;
                    while (r0 < r1 && pyspace(d[r0])) ++r0;
                    uint8_t *copy = c.alloc(r1 - r0 + 1);
                    if (!copy) return;
                    for (uint32_t k = r0; k < r1; ++k) copy[k - r0] = d[k];
                    eval_if(copy, r1 - r0);  // for its errors: never taken
                    if (c.status == ST_UNSUP) c.status = ST_OK;
                    if (c.status) return;
                    inc[depth - 1] = 0;
                    seen[depth - 1] = 0;
                }
            }
            emit_line(nullptr, 0);
            return;
        }
        if (equals("#else")) {
            if (depth) {
                bool taking = !seen[depth - 1] && active(depth - 1);
                inc[depth - 1] = taking;
                seen[depth - 1] = 1;
            }
            emit_line(nullptr, 0);
            return;
        }
        if (equals("#endif")) {
            if (depth) depth--;
            emit_line(nullptr, 0);
            return;
        }
        if (!active(depth)) {
            emit_line(nullptr, 0);
            return;
        }
        if (starts("#define")) {
            for (uint32_t k = 0; k < dn; ++k)
                if (d[k] >= 0x80) { c.set(ST_UNSUP); return; }
            define(d, dn);
            emit_line(nullptr, 0);
            return;
        }
        if (starts("#undef")) {
            undef(d, dn);
            emit_line(nullptr, 0);
            return;
        }
        if (dn && d[0] == '#') {  // #include, #pragma and any other directive
            emit_line(nullptr, 0);
            return;
        }
        text_line(line, n);
    }
};

// _resolve_includes blanking: line.lstrip() matches #\s*include\s+"[^"]+" or
// #\s*include\s+<   (returns 1 for "...", 2 for <...>, 0 otherwise)
__device__ int include_line(const uint8_t *s, uint32_t n) {
    uint32_t i = 0;
    while (i < n && pyspace(s[i])) ++i;
    if (i >= n || s[i] != '#') return 0;
    ++i;
    while (i < n && pyspace(s[i])) ++i;
    const char *w = "include";
    for (int k = 0; k < 7; ++k, ++i)
        if (i >= n || s[i] != (uint8_t)w[k]) return 0;
    uint32_t ws0 = i;
    while (i < n && pyspace(s[i])) ++i;
    if (i == ws0 || i >= n) return 0;
    if (s[i] == '<') return 2;
    if (s[i] != '"') return 0;
    uint32_t j = i + 1;
    while (j < n && s[j] != '"') ++j;
    return (j < n && j > i + 1) ? 1 : 0;
}

struct PPArgs {
    const uint8_t *src;
    const uint64_t *tu_off;
    uint32_t n_tu;
    uint8_t *arena;
    const uint64_t *arena_off;   // n_tu+1 (exclusive scan of arena sizes)
    uint32_t *out_len;           // per TU
    int32_t *status;             // per TU
    uint32_t *qinclude;          // per TU: 1 if a quoted include line was blanked
};

// Arena of a TU of n bytes: output | work A | work B | pool, each region a
// multiple of 16 bytes so every region (and the pool's 16-aligned bump
// allocations, which hold structs with pointers) is suitably aligned.
__host__ __device__ __forceinline__ uint64_t align16(uint64_t x) { return (x + 15) & ~15ull; }
__host__ __device__ __forceinline__ void arena_layout(uint64_t n, uint32_t scale, uint64_t &out,
                                                       uint64_t &work, uint64_t &pool) {
    out = align16(scale * n + 4096);
    work = align16(2 * (scale * n + 4096));
    pool = align16((scale + 4) * n + 65536);
}
__host__ __device__ __forceinline__ uint64_t arena_bytes(uint64_t n, uint32_t scale) {
    uint64_t out, work, pool;
    arena_layout(n, scale, out, work, pool);
    return out + 2 * work + pool;
}

__device__ void preprocess_one(const PPArgs &A, uint32_t t, uint32_t scale) {
    const uint64_t b = A.tu_off[t], e = A.tu_off[t + 1];
    const uint8_t *s = A.src + b;
    const uint32_t n = (uint32_t)(e - b);
    uint8_t *ar = A.arena + A.arena_off[t];
    uint64_t out_cap, wcap, pool_cap;
    arena_layout(n, scale, out_cap, wcap, pool_cap);
    TU u;
    u.c = Ctx{s, n, ar, 0, (uint32_t)out_cap, ar + out_cap, ar + out_cap + wcap, (uint32_t)wcap,
              ar + out_cap + 2 * wcap, 0, (uint32_t)pool_cap, ST_OK};
    u.obj = Dict{};
    u.fn = Dict{};
    u.depth = 0;
    u.first_line = true;
    u.stack = (Frame *)u.c.alloc(sizeof(Frame) * MAX_DEPTH);
    u.tcap = 2 * n + 4096;
    u.tmpl = u.c.alloc(u.tcap);
    uint32_t tw = n + 4096;
    u.t1 = LBuf{u.c.alloc(tw), 0, tw};
    u.t2 = LBuf{u.c.alloc(tw), 0, tw};
    if (u.c.status) {
        A.status[t] = u.c.status;
        A.out_len[t] = 0;
        return;
    }
    // fast path: no '#' and no backslash -> output == input
    bool plain = true;
    for (uint32_t i = 0; i < n && plain; ++i) plain = s[i] != '#' && s[i] != '\\';
    if (plain) {
        for (uint32_t i = 0; i < n; ++i) ar[i] = s[i];
        A.out_len[t] = n;
        A.status[t] = ST_OK;
        return;
    }
    // joined-line buffer: the first half of work buffer A
    LBuf pend{u.c.wa, 0, (uint32_t)wcap};
    bool have_pending = false;
    uint32_t q = 0;
    for (;;) {
        uint32_t r = q;
        while (r < n && s[r] != '\n') ++r;
        // raw line [q, r)
        const uint8_t *L = s + q;
        uint32_t Ln = r - q;
        int inc_kind = include_line(L, Ln);
        if (inc_kind == 1) A.qinclude[t] = 1;
        if (inc_kind) Ln = 0;
        uint32_t rs = Ln;
        while (rs > 0 && pyspace(L[rs - 1])) --rs;
        if (rs > 0 && L[rs - 1] == '\\') {
            if (!pend.append(u.c, L, rs - 1)) break;
            have_pending = true;
        } else {
            if (!pend.append(u.c, L, Ln)) break;
            u.joined_line(pend.p, pend.n);
            pend.n = 0;
            have_pending = false;
            if (u.c.status) break;
        }
        if (r >= n) break;
        q = r + 1;
    }
    if (!u.c.status && have_pending && pend.n > 0) u.joined_line(pend.p, pend.n);
    A.status[t] = u.c.status;
    A.out_len[t] = u.c.status ? 0 : u.c.out_len;
}

__global__ void k_preprocess(PPArgs A, uint32_t scale) {
    uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < A.n_tu) preprocess_one(A, t, scale);
}

// u32 lengths -> u64 (n+1 entries, the last one 0) for the offset scan
__global__ void k_widen_u32(const uint32_t *in, uint64_t *out, uint32_t n) {
    uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) out[t] = in[t];
    if (t == n) out[t] = 0;
}

__global__ void k_pp_arena_sizes(const uint64_t *tu_off, uint32_t n_tu, uint32_t scale,
                                 uint64_t *sizes) {
    uint32_t t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n_tu) sizes[t] = arena_bytes(tu_off[t + 1] - tu_off[t], scale);
    if (t == n_tu) sizes[t] = 0;
}

// Pack each TU's output (at the start of its arena) at out_off[t]; one block
// per TU, 16-byte stores where both sides allow it.
__global__ void k_pp_pack(const uint8_t *arena, const uint64_t *arena_off,
                          const uint64_t *out_off, uint8_t *out, uint32_t n_tu) {
    uint32_t t = blockIdx.x;
    if (t >= n_tu) return;
    const uint8_t *s = arena + arena_off[t];
    uint8_t *d = out + out_off[t];
    uint64_t n = out_off[t + 1] - out_off[t];
    for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) d[i] = s[i];
}

}  // namespace pp
}  // namespace ocb
