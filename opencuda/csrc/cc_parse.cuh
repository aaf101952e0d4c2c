// Parser: tokens -> IR, restating opencuda/frontend/parser.py (the Parser
// class, :31-4448) for the language subset this engine covers.  The reference
// builds SSA IR directly while descending, so value ids, block labels and the
// order of every emitted instruction are side effects of the descent; this
// code follows the same descent function by function, in the same order.
// Constructs outside the subset (structs, unions, typedef/enum definitions,
// __device__ functions, switch, printf, inline asm, ...) mark the TU
// unsupported instead of guessing.
//
// Recursion depth is bounded (MAX_NEST) so the device stack stays bounded.
#pragma once
#include "cc_ir.cuh"

namespace ocb {
namespace cc {

// TokKind values (opencuda/frontend/lexer.py:11-109)
enum : uint32_t {
    TK_INT_LIT = 1, TK_FLOAT_LIT, TK_STRING_LIT, TK_CHAR_LIT, TK_IDENT,
    TK_GLOBAL, TK_SHARED, TK_DEVICE, TK_VOID, TK_INT, TK_UNSIGNED, TK_FLOAT,
    TK_DOUBLE, TK_HALF, TK_CHAR, TK_SHORT, TK_LONG, TK_IF, TK_ELSE, TK_FOR,
    TK_WHILE, TK_RETURN, TK_STRUCT, TK_UNION, TK_TYPEDEF, TK_CONST, TK_CONSTANT,
    TK_VOLATILE, TK_BREAK, TK_CONTINUE, TK_DO, TK_SWITCH, TK_CASE, TK_DEFAULT,
    TK_SIZEOF, TK_ENUM, TK_STATIC, TK_GOTO, TK_BOOL, TK_TRUE, TK_FALSE, TK_SIGNED,
    TK_PLUS, TK_MINUS, TK_STAR, TK_SLASH, TK_PERCENT, TK_AMP, TK_PIPE, TK_CARET,
    TK_TILDE, TK_BANG, TK_LSHIFT, TK_RSHIFT, TK_EQ, TK_NE, TK_LT, TK_LE, TK_GT,
    TK_GE, TK_AND, TK_OR, TK_ASSIGN, TK_PLUS_EQ, TK_MINUS_EQ, TK_STAR_EQ,
    TK_SLASH_EQ, TK_PERCENT_EQ, TK_AMP_EQ, TK_PIPE_EQ, TK_CARET_EQ, TK_LSHIFT_EQ,
    TK_RSHIFT_EQ, TK_LPAREN, TK_RPAREN, TK_LBRACE, TK_RBRACE, TK_LBRACKET,
    TK_RBRACKET, TK_SEMI, TK_COMMA, TK_DOT, TK_ARROW, TK_PLUSPLUS, TK_MINUSMINUS,
    TK_QUESTION, TK_COLON, TK_EOF
};

constexpr int MAX_NEST = 32;

// ---------------------------------------------------------------------------
// An insertion-ordered map name -> operand (a Python dict: assigning an
// existing key keeps its position, del + re-insert moves it to the end).
// ---------------------------------------------------------------------------
struct VarEnt {
    Str name;
    Opnd v;
    uint8_t live;
};
struct VarMap {
    Vec<VarEnt> e;
    Vec<int32_t> ht;  // open addressing over entry indices, -1 empty
    uint32_t live_n;

    OCB_HD void init() {
        e.init();
        ht.init();
        live_n = 0;
    }
    OCB_HD int32_t find(Str k) const {
        if (!ht.n) return -1;
        uint32_t m = ht.n - 1, h = hash(k) & m;
        for (uint32_t i = 0; i <= m; ++i) {
            int32_t x = ht.p[(h + i) & m];
            if (x == -1) return -1;
            if (x >= 0 && e.p[x].live && eq(e.p[x].name, k)) return x;
        }
        return -1;
    }
    OCB_HD OCB_NI void rehash(Arena &a, uint32_t want) {
        uint32_t c = 16;
        while (c < 2 * want + 2) c *= 2;
        ht.init();
        if (!ht.reserve(a, c)) return;
        ht.n = c;
        for (uint32_t i = 0; i < c; ++i) ht.p[i] = -1;
        for (uint32_t i = 0; i < e.n; ++i)
            if (e.p[i].live) {
                uint32_t h = hash(e.p[i].name) & (c - 1);
                while (ht.p[h] != -1) h = (h + 1) & (c - 1);
                ht.p[h] = (int32_t)i;
            }
    }
    OCB_HD Opnd *get(Str k) {
        int32_t x = find(k);
        return x < 0 ? nullptr : &e.p[x].v;
    }
    OCB_HD bool has(Str k) const { return find(k) >= 0; }
    OCB_HD OCB_NI void set(Arena &a, Str k, Opnd v) {
        int32_t x = find(k);
        if (x >= 0) {
            e.p[x].v = v;
            return;
        }
        e.push(a, VarEnt{k, v, 1});
        live_n++;
        if (2 * (e.n + 1) > ht.n) {
            rehash(a, e.n);
        } else {
            uint32_t m = ht.n - 1, h = hash(k) & m;
            while (ht.p[h] >= 0) h = (h + 1) & m;
            ht.p[h] = (int32_t)(e.n - 1);
        }
    }
    OCB_HD void del(Arena &a, Str k) {
        int32_t x = find(k);
        if (x < 0) return;
        e.p[x].live = 0;
        live_n--;
        rehash(a, e.n);
    }
    // dict(self): live entries only, same order
    OCB_HD OCB_NI VarMap copy(Arena &a) const {
        VarMap r;
        r.init();
        r.e.reserve(a, live_n + 1);
        for (uint32_t i = 0; i < e.n; ++i)
            if (e.p[i].live) r.e.push(a, e.p[i]);
        r.live_n = r.e.n;
        r.rehash(a, r.e.n);
        return r;
    }
};

struct Tokens {
    const uint8_t *src;        // batch bytes (token starts are batch offsets)
    const uint32_t *start;     // this TU's tokens
    const uint32_t *kindlen;
    uint32_t n;
};

}  // namespace cc
}  // namespace ocb

namespace ocb {
namespace cc {

enum : int { E_NONE = 0, E_PARSE = 1, E_OTHER = 2 };
// Python exception types, reported as the TU status (OCB_TU_RAISES_*)
enum : int { R_VALUE = 1, R_PARSE = 3, R_KEY = 4, R_OTHER = 6 };

struct SharedInit {  // module-level __shared__ array (name, element type, count)
    Str name;
    Ty ty;
    int64_t count;
};

struct TypedefEnt {
    Str name;
    Ty ty;
};

// A struct name visible to the parser (_struct_types: the latest definition
// of a name wins).
struct StructName {
    Str name;
    Ty ty;
};
// Array members of the struct named `sname` (_struct_field_arrays): base
// name -> element count, for the latest definition that had any.
struct FieldArr {
    Str sname, base;
    uint32_t count;
    uint32_t group;  // entries of one definition share a group number
};
// _inline_struct_return_fields: value id -> {field name -> operand}, kept in
// insertion order per id (dict order decides later bindings).
struct ISRF {
    uint32_t vid;
    Str fname;
    Opnd v;
};

// A __device__ function kept as a token range and expanded at each call
// (parser.py:4031-4087, _device_funcs).
struct DevFunc {
    Str name;
    Ty ret;
    Vec<Param> params;
    uint32_t body_start, body_end;  // the body's '{' ... one past its '}'
};

struct Parser {
    Arena &ar;
    Module &m;
    Tokens tk;
    uint32_t pos;
    int err;              // pending Python exception (E_PARSE = ParseError)
    int nest;             // recursion depth guard
    Kernel *kern;
    uint32_t kidx;
    uint32_t cur;         // current block index
    VarMap vars;
    uint32_t block_count;
    Vec<uint32_t> copy_src;  // by dest id: value index + 1 of its latest identity copy (0 none)
    VarMap row_strides;        // name -> Const index holding the row stride
    VarMap global_consts;      // module-level names bound to constants
    Vec<TypedefEnt> user_typedefs;  // typedef / enum tag names of this TU, in order
    Vec<DevFunc> dfuncs;            // __device__ functions, in definition order
    int32_t inline_dest;            // value receiving `return` inside an inlined body, or -1
    Str inline_merge;               // label that `return` branches to while inlining
    uint32_t inline_depth;
    Vec<SharedInit> module_shared;
    Vec<NameSet> scopes;
    NameSet shared_scalars;
    Vec<Str> break_targets, continue_targets;
    Vec<VarMap> break_snaps, continue_snaps;
    Vec<StructName> snames;        // user struct/union definitions, in order
    Ty vec_types[20];              // built-in vector StructTys, made on first use
    Vec<FieldArr> farrs;
    uint32_t farr_groups;
    Vec<ISRF> isrf;
    Str last_string_lit;           // the last string literal's text (printf format)
    Vec<uint32_t> rec_funcs;       // recursive __device__ functions (dfuncs indices)

    OCB_HD Parser(Arena &a, Module &mod, Tokens t) : ar(a), m(mod), tk(t) {
        pos = 0;
        err = 0;
        nest = 0;
        kern = nullptr;
        kidx = 0;
        cur = 0;
        vars.init();
        block_count = 0;
        copy_src.init();
        row_strides.init();
        global_consts.init();
        user_typedefs.init();
        dfuncs.init();
        inline_dest = -1;
        inline_merge = Str{nullptr, 0};
        inline_depth = 0;
        module_shared.init();
        scopes.init();
        shared_scalars.init();
        break_targets.init();
        continue_targets.init();
        break_snaps.init();
        continue_snaps.init();
        snames.init();
        for (int i = 0; i < 20; ++i) vec_types[i] = 0;
        farrs.init();
        farr_groups = 0;
        isrf.init();
        last_string_lit = Str{"", 0};
        rec_funcs.init();
    }

    // ---- status ----------------------------------------------------------
    OCB_HD bool bad() const { return err || m.unsup || ar.oom; }
    OCB_HD void unsup() { m.unsup = true; }
    // raise <code>: the first exception wins, later ones are never reached
    OCB_HD void raise_(int code) {
        if (!err) {
            err = code == R_PARSE ? E_PARSE : E_OTHER;
            m.raises = code;
        }
    }
    OCB_HD void perr() { raise_(R_PARSE); }
    // `except Exception:` / `except ParseError:` handlers
    OCB_HD bool catch_any() {
        if (!err || m.unsup || ar.oom) return false;
        err = E_NONE;
        m.raises = 0;
        return true;
    }
    OCB_HD bool catch_parse() {
        if (err != E_PARSE || m.unsup || ar.oom) return false;
        err = E_NONE;
        m.raises = 0;
        return true;
    }

    // ---- tokens ------------------------------------------------------------
    OCB_HD uint32_t kind_at(uint32_t i) {
        if (i >= tk.n) {
            raise_(R_OTHER);  // IndexError in the reference
            return TK_EOF;
        }
        return (tk.kindlen[i] >> 24) & 0x7F;  // hex floats: FLOAT_LIT (value in parse_hexfloat)
    }
    OCB_HD Str val_at(uint32_t i) {
        if (i >= tk.n) return Str{"", 0};
        return Str{(const char *)tk.src + tk.start[i], tk.kindlen[i] & 0xFFFFFF};
    }
    OCB_HD uint32_t peek() { return kind_at(pos); }
    OCB_HD Str peekv() { return val_at(pos); }
    OCB_HD uint32_t advance() { return pos++; }
    OCB_HD bool at(uint32_t k) { return peek() == k; }
    OCB_HD bool match(uint32_t k) {
        if (peek() == k) {
            ++pos;
            return true;
        }
        return false;
    }
    OCB_HD bool expect(uint32_t k) {
        if (peek() != k) {
            perr();
            return false;
        }
        ++pos;
        return true;
    }
    OCB_HD bool at_ident_or_soft() {  // IDENT or KW_HALF (_SOFT_KW_AS_IDENT)
        uint32_t k = peek();
        return k == TK_IDENT || k == TK_HALF;
    }
    OCB_HD bool expect_ident(Str &out) {
        if (at_ident_or_soft()) {
            out = peekv();
            ++pos;
            return true;
        }
        perr();
        return false;
    }
    OCB_HD bool is_assign_op(uint32_t k) {
        return k == TK_ASSIGN || k == TK_PLUS_EQ || k == TK_MINUS_EQ || k == TK_STAR_EQ ||
               k == TK_SLASH_EQ || k == TK_PERCENT_EQ || k == TK_AMP_EQ || k == TK_PIPE_EQ ||
               k == TK_CARET_EQ || k == TK_LSHIFT_EQ || k == TK_RSHIFT_EQ;
    }

    // ---- IR helpers ----------------------------------------------------------
    OCB_HD uint32_t new_block(const char *prefix) { return new_block(S(prefix)); }
    OCB_HD uint32_t new_block(Str prefix) {
        block_count++;
        if (!kern) {  // outside a kernel: AttributeError
            raise_(R_OTHER);
            return cur;
        }
        Str lab = cat(ar, prefix, S("_"), utoa(ar, block_count));
        uint32_t b = m.new_block(lab);
        kern->blocks.push(ar, b);
        return b;
    }
    OCB_HD uint32_t new_val(Str name, Ty ty) {
        if (!kern) {  // outside a kernel: AttributeError
            raise_(R_OTHER);
            return m.add_val(0, ty, name);
        }
        return m.add_val(kern->next_id++, ty, name);
    }
    OCB_HD uint32_t new_val(const char *name, Ty ty) { return new_val(S(name), ty); }
    OCB_HD OCB_NI void emit(const Inst &i) {
        if (bad()) return;
        uint32_t ix = m.add_inst(i);
        m.blocks[cur].insts.push(ar, ix);
        // identity copies (dest := src + 0) feed _loop_writeback's ordering
        if (i.kind == I_BIN && i.op == BO_ADD && i.b.k == O_CONST && i.a.k == O_VAL &&
            i.dest >= 0 && const_is_zero(i.b)) {
            uint32_t id = m.vals[i.dest].id;
            if (id >= copy_src.n) {
                if (!copy_src.reserve(ar, id + 1)) return;
                while (copy_src.n <= id) copy_src.p[copy_src.n++] = 0;
            }
            copy_src.p[id] = i.a.x + 1;
        }
    }
    OCB_HD bool const_is_zero(Opnd o) {  // inst.rhs.value == 0 (Python 0 == 0.0)
        const Const &c = m.consts[o.x];
        return c.pyfloat ? c.f == 0.0 : c.i == 0;
    }
    OCB_HD void emit_bin(uint32_t dest, uint8_t op, Opnd a, Opnd b) {
        emit(mk_inst(I_BIN, op, (int32_t)dest, a, b));
    }
    OCB_HD void emit_cmp(uint32_t dest, uint8_t op, Opnd a, Opnd b) {
        emit(mk_inst(I_CMP, op, (int32_t)dest, a, b));
    }
    OCB_HD void emit_load(uint32_t dest, Opnd addr) {
        emit(mk_inst(I_LOAD, 0, (int32_t)dest, addr, onone()));
    }
    OCB_HD void emit_store(Opnd addr, Opnd v) { emit(mk_inst(I_STORE, 0, -1, addr, v)); }
    OCB_HD void emit_cvt(uint32_t dest, Opnd src) {
        emit(mk_inst(I_CVT, 0, (int32_t)dest, src, onone()));
    }
    OCB_HD Block &B() { return m.blocks[cur]; }
    OCB_HD Ty tyof(Opnd o) { return m.opty(o); }
    OCB_HD bool isval(Opnd o) { return o.k == O_VAL; }
    OCB_HD bool iscon(Opnd o) { return o.k == O_CONST; }
    OCB_HD Str vname(Opnd o) { return m.vals[o.x].name; }
    // Value.__eq__ (a dataclass): same name, type and id
    OCB_HD bool val_eq(uint32_t a, uint32_t b) {
        const Value &x = m.vals[a], &y = m.vals[b];
        return x.id == y.id && x.ty == y.ty && eq(x.name, y.name);
    }

    // _const_fold (parser.py:190-235)
    OCB_HD OCB_NI bool const_fold(uint8_t op, Opnd l, Opnd r, Opnd &out) {
        if (!iscon(l) || !iscon(r)) return false;
        const Const a = m.consts[l.x], b = m.consts[r.x];
        bool af = !is_ptr(a.ty) && ty_is_float(a.ty), bf = !is_ptr(b.ty) && ty_is_float(b.ty);
        Ty ty = !is_ptr(a.ty) ? a.ty : (Ty)S_INT32;
        if (bf && !af) ty = b.ty;
        if (af || bf) {
            double x = a.pyfloat ? a.f : (double)a.i, y = b.pyfloat ? b.f : (double)b.i;
            double res;
            switch (op) {
            case BO_ADD: res = x + y; break;
            case BO_SUB: res = x - y; break;
            case BO_MUL: res = x * y; break;
            case BO_DIV: res = y != 0.0 ? x / y : 0.0; break;
            case BO_MOD:
                if (y == 0.0) { res = 0.0; break; }
                unsup();  // Python float % (sign of the divisor): not reproduced
                return false;
            default: return false;
            }
            out = m.cfloat(ty, res);
            return true;
        }
        if (a.pyfloat || b.pyfloat) {  // int(float value): truncation
            unsup();
            return false;
        }
        pyint x = a.i, y = b.i, res = 0;
        bool ok = true;
        switch (op) {
        case BO_ADD: res = x + y; break;
        case BO_SUB: res = x - y; break;
        case BO_MUL: ok = py_mul(x, y, res); break;
        case BO_DIV: {  // C truncation toward zero; x / 0 folds to 0
            if (y == 0) { res = 0; break; }
            pyint q = py_abs(x) / py_abs(y);
            res = ((x >= 0) == (y >= 0)) ? q : -q;
            break;
        }
        case BO_MOD: {
            if (y == 0) { res = 0; break; }
            pyint ax = py_abs(x), ay = py_abs(y);
            res = (ax - (ax / ay) * ay) * (x >= 0 ? 1 : -1);
            break;
        }
        case BO_OR: res = x | y; break;
        case BO_AND: res = x & y; break;
        case BO_XOR: res = x ^ y; break;
        case BO_SHL: ok = py_shl(x, y & 63, res); break;
        case BO_SHR: res = py_shr(x, y & 63); break;
        default: return false;
        }
        if (!ok || !py_ok(res)) {  // a Python int beyond the kept range
            unsup();
            return false;
        }
        out = m.cint(ty, res);
        return true;
    }
    OCB_HD static bool mul_ovf_(int64_t x, int64_t y, int64_t &r) {
        if (x == 0 || y == 0) { r = 0; return false; }
        if ((x == -1 && y == INT64_MIN) || (y == -1 && x == INT64_MIN)) return true;
        int64_t p = (int64_t)((uint64_t)x * (uint64_t)y);
        if (p / y != x) return true;
        r = p;
        return false;
    }

    // _result_type (parser.py:841-872)
    OCB_HD Ty result_type(Opnd a, Opnd b) {
        Ty at = tyof(a), bt = tyof(b);
        if (at == S_BOOL) at = S_INT32;
        if (bt == S_BOOL) bt = S_INT32;
        bool af = ty_is_float(at), bf = ty_is_float(bt);
        if (af || bf) {
            if (af && bf) return ty_size(at) >= ty_size(bt) ? at : bt;
            return af ? at : bt;
        }
        if (is_ptr(at)) return at;
        if (is_ptr(bt)) return bt;
        if (ty_size(at) == 8 || ty_size(bt) == 8) return ty_size(at) == 8 ? at : bt;
        if (ty_size(at) == ty_size(bt) && ty_is_signed(at) != ty_is_signed(bt))
            return ty_is_signed(at) ? bt : at;
        return at;
    }

    // _scale_ptr_arith_offset (parser.py:237-254)
    OCB_HD Opnd scale_ptr_off(Ty ptr_ty, Opnd v) {
        uint32_t es = m.tsize(ty_pointee(ptr_ty));
        if (es == 1) return v;
        Ty it = (isval(v) || iscon(v)) ? tyof(v) : (Ty)S_INT32;
        if (iscon(v)) {
            const Const c = m.consts[v.x];
            if (c.pyfloat) { unsup(); return v; }
            pyint r;
            if (!py_mul(c.i, es, r)) { unsup(); return v; }
            return m.cint(it, r);
        }
        uint32_t s = new_val("ptr_off", it);
        emit_bin(s, BO_MUL, v, m.cint(it, es));
        return ov(s);
    }

    // str.replace(a, b) (all non-overlapping occurrences, left to right)
    OCB_HD Str str_replace(Str s, const char *a, const char *b) {
        uint32_t na = cstrlen(a), nb = cstrlen(b), cnt = 0;
        for (uint32_t i = 0; i + na <= s.n;) {
            if (mem_eq(s.p + i, a, na)) {
                cnt++;
                i += na;
            } else {
                i++;
            }
        }
        if (!cnt) return s;
        char *d = (char *)ar.alloc(s.n + cnt * nb + 1, 1);
        if (!d) return s;
        uint32_t k = 0;
        for (uint32_t i = 0; i < s.n;) {
            if (i + na <= s.n && mem_eq(s.p + i, a, na)) {
                for (uint32_t j = 0; j < nb; ++j) d[k++] = b[j];
                i += na;
            } else {
                d[k++] = s.p[i++];
            }
        }
        d[k] = 0;
        return Str{d, k};
    }
    // a string literal token as the parser keeps it (parser.py:2203-2209):
    // the quotes dropped, then \n, \t, \r, \\ and \" replaced in that order
    OCB_HD Str string_lit_text(Str tokv) {
        Str raw{tokv.p + 1, tokv.n >= 2 ? tokv.n - 2 : 0};
        raw = str_replace(raw, "\\n", "\n");
        raw = str_replace(raw, "\\t", "\t");
        raw = str_replace(raw, "\\r", "\r");
        raw = str_replace(raw, "\\\\", "\\");
        raw = str_replace(raw, "\\\"", "\"");
        return raw;
    }

    // int(const.value) of an array dimension (1 for a non-constant); float
    // dimensions are outside the subset
    OCB_HD bool const_dim_of(Opnd o, int64_t &out) {
        if (o.k != O_CONST) {
            out = 1;
            return true;
        }
        const Const &c = m.consts[o.x];
        if (c.pyfloat || c.i > INT64_MAX / 2 || c.i < INT64_MIN / 2) {
            unsup();
            return false;
        }
        out = (int64_t)c.i;
        return true;
    }
    // int(const.value) % n (Python modulo, n > 0)
    OCB_HD bool const_mod(Opnd o, uint32_t n, int64_t &k) {
        const Const &c = m.consts[o.x];
        if (c.pyfloat) {
            unsup();
            return false;
        }
        pyint r = c.i % (pyint)n;
        if (r < 0) r += n;
        k = (int64_t)r;
        return true;
    }

    // _loop_writeback (parser.py:256-364)
    OCB_HD Opnd chain_src(uint32_t id) {
        if (id < copy_src.n && copy_src.p[id]) return ov(copy_src.p[id] - 1);
        return onone();
    }
    OCB_HD Opnd root(Opnd v) {
        // follow identity copies by value id; stop on a repeat
        uint32_t seen[64];
        uint32_t ns = 0;
        while (v.k == O_VAL) {
            uint32_t id = m.vals[v.x].id;
            for (uint32_t i = 0; i < ns; ++i)
                if (seen[i] == id) return v;
            if (ns < 64) seen[ns++] = id;
            else { unsup(); return v; }
            Opnd s = chain_src(id);
            if (s.k == O_NONE) break;
            v = s;
        }
        return v;
    }
    OCB_HD OCB_NI void loop_writeback(VarMap &entry) {
        struct P { Str name; uint32_t ev; Opnd cv; };
        Vec<P> pending, ordered;
        pending.init();
        ordered.init();
        // pass 1: struct sentinels get their entry binding back, nothing emitted
        for (uint32_t i = 0; i < entry.e.n; ++i) {
            const VarEnt &en = entry.e[i];
            if (!en.live || en.v.k != O_VAL || !ty_is_struct(m.vals[en.v.x].ty)) continue;
            Opnd *c = vars.get(en.name);
            if (!c || c->k != O_VAL || c->x != en.v.x) vars.set(ar, en.name, en.v);
        }
        for (uint32_t i = 0; i < entry.e.n; ++i) {
            const VarEnt &en = entry.e[i];
            if (!en.live || en.v.k != O_VAL) continue;
            if (ty_is_struct(m.vals[en.v.x].ty)) continue;
            Opnd *c = vars.get(en.name);
            if (!c) continue;
            if (c->k == O_VAL && c->x == en.v.x) continue;  // `is`
            if (c->k == O_VAL && ty_is_struct(m.vals[c->x].ty)) continue;
            if (c->k == O_VAL || c->k == O_CONST) pending.push(ar, P{en.name, en.v.x, *c});
        }
        // sequence the copies so no copy clobbers another's source
        uint32_t guard = pending.n * pending.n + pending.n + 1, iters = 0;
        while (pending.n) {
            if (++iters > guard) break;
            uint32_t safe = 0xFFFFFFFFu;
            for (uint32_t i = 0; i < pending.n && safe == 0xFFFFFFFFu; ++i) {
                bool clob = false;
                for (uint32_t j = 0; j < pending.n && !clob; ++j) {
                    if (j == i) continue;
                    Opnd r = root(pending[j].cv);
                    if (r.k == O_VAL && r.x == pending[i].ev) clob = true;
                }
                if (!clob) safe = i;
            }
            if (safe == 0xFFFFFFFFu) safe = 0;
            ordered.push(ar, pending[safe]);
            pending.erase(safe);
        }
        // the order is fixed before any copy is emitted (emitting extends the chain)
        for (uint32_t i = 0; i < ordered.n; ++i) {
            const P &p = ordered[i];
            emit_bin(p.ev, BO_ADD, p.cv, m.cint(m.vals[p.ev].ty, 0));
            vars.set(ar, p.name, ov(p.ev));
        }
    }
    OCB_HD void declare_local(Str name) {
        if (scopes.n) scopes.back().add(ar, name);
    }

    // ---- declared here, defined in cc_parse_expr.cuh / cc_parse_stmt.cuh ----
    OCB_HD OCB_NI bool parse_type(Ty &out);
    OCB_HD OCB_NI bool parse_type_with_ptr(Ty &out);
    OCB_HD OCB_NI Opnd parse_expr();
    OCB_HD OCB_NI Opnd parse_assign_expr();
    OCB_HD OCB_NI Opnd parse_or_expr();
    OCB_HD OCB_NI Opnd parse_and_expr();
    OCB_HD OCB_NI Opnd parse_bitor_expr();
    OCB_HD OCB_NI Opnd parse_bitxor_expr();
    OCB_HD OCB_NI Opnd parse_bitand_expr();
    OCB_HD OCB_NI Opnd parse_cmp_expr();
    OCB_HD OCB_NI Opnd parse_shift_expr();
    OCB_HD OCB_NI Opnd parse_add_expr();
    OCB_HD OCB_NI Opnd parse_mul_expr();
    OCB_HD OCB_NI Opnd parse_unary_expr();
    OCB_HD OCB_NI Opnd parse_postfix_expr();
    OCB_HD OCB_NI Opnd parse_primary_expr();
    OCB_HD OCB_NI Opnd parse_call(Str name);
    OCB_HD OCB_NI Opnd parse_lvalue_or_expr();
    OCB_HD OCB_NI void parse_stmt();
    OCB_HD OCB_NI void parse_stmt_inner();
    OCB_HD OCB_NI void parse_stmt_or_block();
    OCB_HD OCB_NI void pop_scope(NameSet &inner, VarMap &outer);
    OCB_HD void push_loop(Str brk, Str cont, VarMap &snap);
    OCB_HD void pop_loop();
    OCB_HD OCB_NI void parse_while();
    OCB_HD OCB_NI void parse_do();
    OCB_HD OCB_NI void parse_enum_def();
    OCB_HD OCB_NI void parse_typedef();
    // a typedef of this TU (the latest binding of the name wins, as a dict
    // assignment does in the reference)
    OCB_HD bool user_typedef(Str v, Ty &t) const {
        for (uint32_t i = user_typedefs.n; i-- > 0;)
            if (eq(user_typedefs[i].name, v)) {
                t = user_typedefs[i].ty;
                return true;
            }
        return false;
    }
    OCB_HD void add_typedef(Str v, Ty t) { user_typedefs.push(ar, TypedefEnt{v, t}); }
    // ---- structs (cc_parse_struct.cuh) ----
    OCB_HD OCB_NI bool vector_type(Str v, Ty &t);
    OCB_HD bool user_struct(Str v, Ty &t) const {
        for (uint32_t i = snames.n; i-- > 0;)
            if (eq(snames[i].name, v)) {
                t = snames[i].ty;
                return true;
            }
        return false;
    }
    // name in self._struct_types (user definitions, then the vector types)
    OCB_HD bool find_struct(Str v, Ty &t) { return user_struct(v, t) || vector_type(v, t); }
    // name in self._typedefs or name in self._struct_types
    OCB_HD bool is_type_name(Str v);
    OCB_HD OCB_NI bool parse_struct_def(Ty &out);
    // _struct_field_arrays.get(sty.name, {}).get(member): element count or 0
    OCB_HD uint32_t field_array(Ty st, Str member);
    OCB_HD bool isstruct(Opnd o) { return o.k == O_VAL && ty_is_struct(tyof(o)); }
    OCB_HD bool isptr_struct(Opnd o) {
        return o.k == O_VAL && is_ptr(tyof(o)) && ty_is_struct(ty_pointee(tyof(o)));
    }
    // ScalarTy instance test (not a pointer, not a struct)
    OCB_HD static bool is_scalar_ty(Ty t) { return !is_ptr(t) && !ty_is_struct(t); }
    OCB_HD int32_t isrf_find(uint32_t vid, Str f) const {
        for (uint32_t i = 0; i < isrf.n; ++i)
            if (isrf[i].vid == vid && eq(isrf[i].fname, f)) return (int32_t)i;
        return -1;
    }
    OCB_HD bool isrf_has(uint32_t vid) const {
        for (uint32_t i = 0; i < isrf.n; ++i)
            if (isrf[i].vid == vid) return true;
        return false;
    }
    OCB_HD void isrf_set(uint32_t vid, Str f, Opnd v) {
        int32_t i = isrf_find(vid, f);
        if (i >= 0) isrf[i].v = v;
        else isrf.push(ar, ISRF{vid, f, v});
    }
    // the field's value of a struct value: the per-field map of its id, else
    // the variable `<name>_<field>` (or onone())
    OCB_HD Opnd struct_field_src(uint32_t sval, Str f) {
        int32_t i = isrf_find(m.vals[sval].id, f);
        if (i >= 0) return isrf[i].v;
        Opnd *o = vars.get(cat(ar, m.vals[sval].name, S("_"), f));
        return o ? *o : onone();
    }
    // field index of `member` in struct type st, raising KeyError when absent
    OCB_HD int32_t field_or_raise(Ty st, Str member) {
        int32_t fi = m.field_index(st, member);
        if (fi < 0) raise_(R_KEY);
        return fi;
    }
    OCB_HD OCB_NI void zero_init_fields(Str prefix, Ty st);
    OCB_HD OCB_NI void load_struct_fields(Opnd base, Ty st, Str prefix, uint32_t abs_off,
                                          uint32_t as, bool ptr_fields, bool declare_nested);
    OCB_HD OCB_NI void copy_struct_fields(uint32_t rhs, Str update_name);
    OCB_HD OCB_NI Opnd member_of_ptr(Opnd lhs, Str member);
    OCB_HD OCB_NI Opnd member_of_struct(Opnd lhs, Str member, Str &src_name);
    OCB_HD OCB_NI Opnd parse_compound_literal(Ty st);
    OCB_HD OCB_NI Opnd field_addr(Opnd addr, Str member);
    OCB_HD OCB_NI Opnd field_chain(Opnd addr, Ty cur_ty, uint32_t as);
    OCB_HD OCB_NI Opnd member_lvalue(Opnd var);
    OCB_HD OCB_NI void flat_struct_params(Str prefix, Ty st, uint32_t slot, NameSet &seen,
                                          uint32_t &next);
    OCB_HD OCB_NI Opnd spill_scalar(Str name, Opnd value);
    OCB_HD OCB_NI void parse_device_func();
    OCB_HD OCB_NI Opnd inline_call(uint32_t fi, Vec<Opnd> &args, Str name);
    OCB_HD OCB_NI bool recursive_funcs(Vec<uint32_t> &out);
    OCB_HD OCB_NI void compile_devfn(uint32_t fi);
    // a name in the reference's _recursive_device_funcs
    OCB_HD bool is_recursive(Str v) const {
        for (uint32_t i = 0; i < rec_funcs.n; ++i)
            if (eq(dfuncs[rec_funcs[i]].name, v)) return true;
        return false;
    }
    // the definition a call resolves to (a later definition replaces an
    // earlier one, as a dict assignment does)
    OCB_HD int32_t find_dfunc(Str v) const {
        for (uint32_t i = dfuncs.n; i-- > 0;)
            if (eq(dfuncs[i].name, v)) return (int32_t)i;
        return -1;
    }
    OCB_HD OCB_NI void parse_switch();
    OCB_HD OCB_NI void parse_asm();
    OCB_HD OCB_NI void parse_decl(Ty ty, bool vol);
    OCB_HD OCB_NI void parse_shared(bool vol);
    OCB_HD OCB_NI void parse_if();
    OCB_HD OCB_NI void parse_for();
    OCB_HD OCB_NI void parse_expr_stmt();
    OCB_HD OCB_NI void parse_kernel();
    OCB_HD OCB_NI void parse_module();
    OCB_HD OCB_NI void parse_gvar(bool constant_form);
    OCB_HD Opnd gaddr(uint32_t g);
};

}  // namespace cc
}  // namespace ocb
