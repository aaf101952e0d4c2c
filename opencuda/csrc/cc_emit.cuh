// PTX emitter: restates opencuda/codegen/emit.py (the linear-scan register
// allocator _build_alloc_map :115-342, PTXEmitter.emit_kernel :648-1126,
// _emit_block/_emit_inst/_emit_term :1129-3123) and the module assembly of
// ir_to_ptx :3126 + the CLI's --emit-ptx text (__main__.py:60-85) for the
// subset of IR this engine builds.  The reference emits text lines and then
// rewrites them with regular-expression peepholes; this code keeps the same
// line-level representation and restates each peephole's pattern by hand.
#pragma once
#include "cc_opt_base.cuh"

namespace ocb {
namespace cc {

// ---------------------------------------------------------------------------
// text building
// ---------------------------------------------------------------------------
struct SB {  // growable string in the arena
    Arena *a;
    char *p;
    uint32_t n, cap;
    OCB_HD void init(Arena &ar, uint32_t c = 64) {
        a = &ar;
        cap = c;
        n = 0;
        p = (char *)ar.alloc(cap, 1);
        if (!p) cap = 0;
    }
    OCB_HD void grow(uint32_t need) {
        uint32_t nc = cap ? cap * 2 : 64;
        while (nc < need) nc *= 2;
        char *np = (char *)a->alloc(nc, 1);
        if (!np) {
            cap = n;
            return;
        }
        for (uint32_t i = 0; i < n; ++i) np[i] = p[i];
        p = np;
        cap = nc;
    }
    OCB_HD SB &c(char ch) {
        if (n + 1 > cap) grow(n + 1);
        if (n < cap) p[n++] = ch;
        return *this;
    }
    OCB_HD SB &s(const char *z) {
        while (*z) c(*z++);
        return *this;
    }
    OCB_HD SB &s(Str z) {
        if (n + z.n > cap) grow(n + z.n);
        for (uint32_t i = 0; i < z.n && n < cap; ++i) p[n++] = z.p[i];
        return *this;
    }
    OCB_HD SB &i(pyint v) {
        char t[48];
        int k = 0;
        unsigned __int128 u = v < 0 ? (unsigned __int128)0 - (unsigned __int128)v : (unsigned __int128)v;
        do {
            t[k++] = (char)('0' + (int)(u % 10));
            u /= 10;
        } while (u);
        if (v < 0) c('-');
        while (k) c(t[--k]);
        return *this;
    }
    OCB_HD SB &hex(uint64_t v, int digits) {  // upper-case, zero padded
        const char *h = "0123456789ABCDEF";
        for (int q = digits - 1; q >= 0; --q) c(h[(v >> (4 * q)) & 15]);
        return *this;
    }
    OCB_HD Str str() const { return Str{p, n}; }
};

OCB_HD inline bool is_wsc(char c) {  // \s for the ASCII text emitted here
    return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\f' || c == '\v' ||
           (c >= 0x1c && c <= 0x1f);
}
OCB_HD inline bool is_wc(char c) {  // \w (ASCII; names outside ASCII are declined)
    return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_';
}
OCB_HD inline bool is_dg(char c) { return c >= '0' && c <= '9'; }

// cursor helpers for the hand-written patterns
struct Cur {
    Str s;
    uint32_t i;
    OCB_HD bool end() const { return i >= s.n; }
    OCB_HD char ch() const { return i < s.n ? s.p[i] : 0; }
    OCB_HD bool ws1() {  // \s+
        uint32_t j = i;
        while (j < s.n && is_wsc(s.p[j])) ++j;
        if (j == i) return false;
        i = j;
        return true;
    }
    OCB_HD void ws0() {  // \s*
        while (i < s.n && is_wsc(s.p[i])) ++i;
    }
    OCB_HD bool lit(const char *z) {
        uint32_t j = i;
        for (; *z; ++z, ++j)
            if (j >= s.n || s.p[j] != *z) return false;
        i = j;
        return true;
    }
    OCB_HD bool word(Str &out) {  // \w+
        uint32_t j = i;
        while (j < s.n && is_wc(s.p[j])) ++j;
        if (j == i) return false;
        out = Str{s.p + i, j - i};
        i = j;
        return true;
    }
    OCB_HD bool reg(Str &out) {  // %\w+
        if (ch() != '%') return false;
        uint32_t save = i;
        ++i;
        Str w;
        if (!word(w)) {
            i = save;
            return false;
        }
        out = Str{s.p + save, i - save};
        return true;
    }
    OCB_HD bool digits(Str &out) {
        uint32_t j = i;
        while (j < s.n && is_dg(s.p[j])) ++j;
        if (j == i) return false;
        out = Str{s.p + i, j - i};
        i = j;
        return true;
    }
    OCB_HD bool nonws(Str &out) {  // \S+
        uint32_t j = i;
        while (j < s.n && !is_wsc(s.p[j])) ++j;
        if (j == i) return false;
        out = Str{s.p + i, j - i};
        i = j;
        return true;
    }
};

// ---------------------------------------------------------------------------
// types -> PTX spellings (emit.py:20-112)
// ---------------------------------------------------------------------------
OCB_HD inline const char *ptx_type(Ty t) {
    if (is_ptr(t)) return "u64";
    switch (ty_scalar(t)) {
    case S_INT8: return "s8";
    case S_UINT8: return "u8";
    case S_INT16: return "s16";
    case S_UINT16: return "u16";
    case S_INT32: return "s32";
    case S_UINT32: return "u32";
    case S_INT64: return "s64";
    case S_UINT64: return "u64";
    case S_FLOAT: return "f32";
    case S_DOUBLE: return "f64";
    case S_HALF: return "f16";
    default: return "u32";  // void, bool
    }
}
OCB_HD inline bool cstr_eq(const char *a, const char *b) {
    while (*a && *a == *b) ++a, ++b;
    return *a == *b;
}
OCB_HD inline bool cstr_in(const char *a, const char *l) { return in_list(S(a), l); }
OCB_HD inline const char *ptx_mov_type(Ty t) {
    const char *p = ptx_type(t);
    if (cstr_in(p, " s8 u8 s16 u16 ")) return "b32";
    if (cstr_eq(p, "f16")) return "b16";
    return p;
}
enum : int { PF_R = 0, PF_RD, PF_F, PF_FD, PF_H, PF_P, PF_N };
OCB_HD inline const char *pf_name(int p) {
    const char *n[] = {"r", "rd", "f", "fd", "h", "p"};
    return n[p];
}
OCB_HD inline int reg_prefix(Ty t) {
    if (is_ptr(t)) return PF_RD;
    uint32_t s = ty_scalar(t);
    if (s == S_HALF) return PF_H;
    if (s == S_DOUBLE) return PF_FD;
    if (ty_size(t) == 8) return PF_RD;
    if (ty_is_float(t)) return PF_F;
    return PF_R;
}
OCB_HD inline bool is_half(Ty t) { return !is_ptr(t) && ty_scalar(t) == S_HALF; }
OCB_HD inline bool is_64bit(Ty t) { return is_ptr(t) || ty_size(t) == 8; }
// _cvt_modifier (emit.py:95-112)
OCB_HD inline const char *cvt_modifier(Ty dst, Ty src) {
    bool df = ty_is_float(dst), sf = ty_is_float(src);
    bool di = !is_ptr(dst) && !df, si = !is_ptr(src) && !sf;
    if (sf && di) return ".rzi";
    if (si && df) return ".rn";
    if (sf && df && ty_size(dst) < ty_size(src)) return ".rn";
    return "";
}

// struct.pack('>f', x): the float32 bits, false when Python raises OverflowError
OCB_HD inline bool pack_f32(double x, uint32_t &bits) {
    float y = (float)x;
    if ((y - y != 0.0f) && (x - x == 0.0)) return false;  // finite rounds to inf
    memcpy(&bits, &y, 4);
    return true;
}
// struct.pack('>e', x): IEEE half, round half to even; false on overflow
OCB_HD inline bool pack_f16(double x, uint16_t &bits) {
    uint64_t d;
    memcpy(&d, &x, 8);
    uint16_t sign = (uint16_t)((d >> 48) & 0x8000);
    uint64_t mag = d & 0x7FFFFFFFFFFFFFFFull;
    if (mag >= 0x7FF0000000000000ull) {  // inf / nan
        if (mag == 0x7FF0000000000000ull) bits = sign | 0x7C00;
        else bits = sign | 0x7E00;
        return true;
    }
    double ax = x < 0 ? -x : x;
    if (ax == 0.0) {
        bits = sign;
        return true;
    }
    // scale to an integer count of the smallest half step where it applies
    int e;
    double m = frexp(ax, &e);  // ax = m * 2^e, m in [0.5, 1)
    // half: normal exponent range 2^-14 .. 2^15, 10 fraction bits
    if (e > 16) return false;
    double q;
    int exp_field;
    if (e <= -14) {  // subnormal: units of 2^-24
        q = ldexp(ax, 24);
        exp_field = 0;
    } else {
        q = ldexp(m, 11);  // 11 significant bits, value in [1024, 2048)
        exp_field = e - 1 + 15;
    }
    double fl = floor(q);
    double fr = q - fl;
    uint64_t iq = (uint64_t)fl;
    if (fr > 0.5 || (fr == 0.5 && (iq & 1))) iq++;
    uint32_t out;
    if (exp_field == 0) {
        out = (uint32_t)iq;  // may carry into the first normal exponent
    } else {
        if (iq == 2048) {
            iq = 1024;
            exp_field++;
        }
        if (exp_field >= 31) return false;
        out = ((uint32_t)exp_field << 10) | (uint32_t)(iq - 1024);
    }
    bits = sign | (uint16_t)out;
    return true;
}

// ---------------------------------------------------------------------------
// the emitter of one TU
// ---------------------------------------------------------------------------
struct Emit {
    Module &m;
    Arena &ar;
    Arena &tmp;
    Kernel *k;
    bool fail;  // an exception in the reference or a construct outside the subset
    // allocation (per kernel), indexed by value id
    uint32_t nid0;
    int32_t *alloc;       // phys or -1
    int32_t *fb_alloc;    // fallback phys or -1 (grown on demand)
    uint32_t fb_cap;
    uint8_t *pred;        // pred ids (grows)
    uint32_t pred_cap;
    int alloc_max[PF_N], fb_count[PF_N], reg_counts[PF_N];
    int32_t *widen;       // id -> value index of the widened copy, -1
    uint32_t widen_cap;
    Vec<Str> *lines;      // current output lines
    LabelSet skip;
    Vec<Str> preamble;    // module preamble (ir_to_ptx)
    int term_depth;       // nesting of _emit_term through inlined merge blocks
    // printf (emit.py:681-694, :1110-1125, :1661-1740)
    struct PFmt {
        Str label, fmt;
    };
    Vec<PFmt> pfs;        // this kernel's format strings, in block order
    uint32_t pf_idx;      // the next one an emitted printf takes
    uint32_t pf_count;    // printf calls emitted in this kernel
    bool vprintf_decl;    // the module preamble declares vprintf
    Vec<Str> fmt_done;    // format labels already in the module preamble
    // per kernel, by label: the last block with it and the number of blocks
    // whose terminator targets it (built on first use; terminators do not
    // change while a kernel is emitted)
    struct LblEnt {
        Str l;
        int32_t blk;
        uint32_t preds;
    };
    LblEnt *lt;
    uint32_t lt_cap;
    bool lt_ok;

    OCB_HD Emit(Module &mod, Arena &tmp_) : m(mod), ar(*mod.ar), tmp(tmp_), k(nullptr), fail(false) {
        preamble.init();
        term_depth = 0;
        pfs.init();
        pf_idx = pf_count = 0;
        vprintf_decl = false;
        fmt_done.init();
        lt = nullptr;
        lt_cap = 0;
        lt_ok = false;
    }
#ifdef OCB_TRAP_UNSUP
    void unsup(int line = __builtin_LINE()) {
        fprintf(stderr, "emit unsupported at line %d\n", line);
        fail = true;
        m.unsup = true;
    }
#else
    OCB_HD void unsup() { fail = true; m.unsup = true; }
#endif
    OCB_HD bool bad() const { return fail || m.unsup || ar.oom || tmp.oom; }
    // the reference raises here (OverflowError from struct.pack, ...): the TU's
    // status becomes that exception
    OCB_HD void raise_(int code) {
        if (!fail) m.raises = code;
        fail = true;
    }
    OCB_HD Inst &I(uint32_t ix) { return m.insts[ix]; }
    OCB_HD Block &B(uint32_t b) { return m.blocks[b]; }
    OCB_HD const Value &V(uint32_t vx) const { return m.vals[vx]; }
    OCB_HD uint32_t vid(Opnd o) const { return m.vals[o.x].id; }
    OCB_HD SB sb() {
        SB b;
        b.init(ar);
        return b;
    }
    OCB_HD void put(SB &b) { lines->push(ar, b.str()); }
    OCB_HD void put(const char *z) { lines->push(ar, S(z)); }
    OCB_HD uint32_t new_value(Str name, Ty ty) { return m.add_val(k->next_id++, ty, name); }
    OCB_HD uint32_t new_value(const char *name, Ty ty) { return new_value(S(name), ty); }
    OCB_HD Str nm(const char *a, pyint n) {  // f"{a}{n}"
        SB b = sb();
        b.s(a).i(n);
        return b.str();
    }
    OCB_HD Str nm2(const char *a, pyint n, const char *c, pyint d) {
        SB b = sb();
        b.s(a).i(n).s(c).i(d);
        return b.str();
    }

    // ---- id-indexed tables that grow with emission-time values ------------
    template <class T>
    OCB_HD bool grow_arr(T *&p, uint32_t &cap, uint32_t need, T fill) {
        if (need < cap) return true;
        uint32_t nc = cap ? cap : 64;
        while (nc <= need) nc *= 2;
        T *np = (T *)tmp.alloc(sizeof(T) * (uint64_t)nc, 16);
        if (!np) return false;
        for (uint32_t i = 0; i < cap; ++i) np[i] = p[i];
        for (uint32_t i = cap; i < nc; ++i) np[i] = fill;
        p = np;
        cap = nc;
        return true;
    }
    OCB_HD bool is_pred(uint32_t id) const { return id < pred_cap && pred[id]; }
    OCB_HD void add_pred(uint32_t id) {
        if (!grow_arr(pred, pred_cap, id, (uint8_t)0)) { unsup(); return; }
        pred[id] = 1;
    }

    // ---- _reg / _operand (emit.py:363-417) ----------------------------------
    OCB_HD Str reg_name(int pf, int phys) {
        SB b = sb();
        b.c('%').s(pf_name(pf)).i(phys);
        return b.str();
    }
    OCB_HD Str reg(uint32_t vx) {
        const Value &v = V(vx);
        int pf = is_pred(v.id) ? PF_P : reg_prefix(v.ty);
        int phys;
        if (v.id < nid0 && alloc[v.id] >= 0) {
            phys = alloc[v.id];
        } else {
            if (!grow_arr(fb_alloc, fb_cap, v.id, (int32_t)-1)) { unsup(); return S("%r0"); }
            if (fb_alloc[v.id] >= 0) {
                phys = fb_alloc[v.id];
            } else {
                phys = alloc_max[pf] + fb_count[pf];
                fb_count[pf]++;
                fb_alloc[v.id] = phys;
            }
        }
        if (reg_counts[pf] < phys + 1) reg_counts[pf] = phys + 1;
        return reg_name(pf, phys);
    }
    OCB_HD Str reg(Opnd o) { return reg(o.x); }
    OCB_HD Str alloc_pred() {  // _alloc_pred
        int idx = alloc_max[PF_P] + fb_count[PF_P];
        fb_count[PF_P]++;
        if (reg_counts[PF_P] < idx + 1) reg_counts[PF_P] = idx + 1;
        return reg_name(PF_P, idx);
    }
    OCB_HD Str fresh_pred() {  // p_idx = _reg_counts.get('p', 0); += 1
        int idx = reg_counts[PF_P];
        reg_counts[PF_P] = idx + 1;
        return reg_name(PF_P, idx);
    }
    OCB_HD Str konst(Opnd o, const char *force) {
        const Const &c = m.consts[o.x];
        PyVal v = pv_of(c);
        bool is_f64 = force ? cstr_eq(force, "f64") : (ty_is_float(c.ty) && ty_size(c.ty) == 8);
        bool is_fp = force ? (cstr_eq(force, "f32") || cstr_eq(force, "f64")) : ty_is_float(c.ty);
        bool is_h = force && cstr_eq(force, "f16");
        SB b = sb();
        if (is_h) {
            uint16_t bits;
            if (!pack_f16(pv_to_float(v), bits)) { raise_(2); return S("0"); }
            b.s("0h").hex(bits, 4);
            return b.str();
        }
        if (is_f64) {
            double f = pv_to_float(v);
            uint64_t bits;
            memcpy(&bits, &f, 8);
            b.s("0d").hex(bits, 16);
            return b.str();
        }
        if (is_fp) {
            uint32_t bits;
            if (!pack_f32(pv_to_float(v), bits)) { raise_(2); return S("0"); }
            b.s("0f").hex(bits, 8);
            return b.str();
        }
        pyint iv;
        if (!pv_to_int(v, iv)) {
            if (v.isf && v.f != v.f) raise_(1);                    // int(nan): ValueError
            else if (v.isf && !is_finite(v.f)) raise_(2);          // int(inf): OverflowError
            else unsup();
            return S("0");
        }
        b.i(iv);
        return b.str();
    }
    // _operand(op, force_type, kernel); with_kernel selects the predicate path
    OCB_HD Str opnd(Opnd o, const char *force = nullptr, bool with_kernel = false) {
        if (o.k == O_VAL) {
            if (with_kernel && is_pred(vid(o)) && force && !cstr_eq(force, "pred"))
                return pred_to_int(o, force);
            return reg(o);
        }
        if (o.k == O_CONST) return konst(o, force);
        if (o.k == O_SYM) return m.gvars[o.x].name;  // the symbol as an address
        unsup();
        return S("?");
    }
    OCB_HD Str pred_to_int(Opnd o, const char *dest_ty) {
        uint32_t t = new_value(nm("_pred_int_", vid(o)), S_INT32);
        SB b = sb();
        Str tr = reg(t);
        b.s("    selp.").s(dest_ty).c(' ').s(tr).s(", 1, 0, ").s(reg(o)).c(';');
        put(b);
        return tr;
    }
    OCB_HD Str coerce_to_float(Opnd o, const char *fty) {
        if (o.k == O_CONST) return opnd(o, fty);
        if (o.k != O_VAL) { unsup(); return S("?"); }
        Ty t = V(o.x).ty;
        const char *op = is_ptr(t) ? nullptr : ptx_type(t);
        if (op && cstr_eq(op, fty)) return reg(o);
        Ty dt = cstr_eq(fty, "f64") ? (Ty)S_DOUBLE : cstr_eq(fty, "f16") ? (Ty)S_HALF : (Ty)S_FLOAT;
        uint32_t tv = new_value(nm("_coerce_", vid(o)), dt);
        SB b = sb();
        if (op && cstr_eq(op, "f16") && cstr_eq(fty, "f32")) {
            Str tr = reg(tv);
            b.s("    cvt.f32.f16 ").s(tr).s(", ").s(reg(o)).c(';');
        } else if (op && cstr_eq(op, "f16") && cstr_eq(fty, "f64")) {
            Str tr = reg(tv);
            b.s("    cvt.f64.f16 ").s(tr).s(", ").s(reg(o)).c(';');
        } else if (op && (cstr_eq(op, "s32") || cstr_eq(op, "u32")) && cstr_eq(fty, "f32")) {
            Str tr = reg(tv);
            b.s("    cvt.rn.f32.").s(op).c(' ').s(tr).s(", ").s(reg(o)).c(';');
        } else if (op && (cstr_eq(op, "s32") || cstr_eq(op, "u32")) && cstr_eq(fty, "f64")) {
            Str tr = reg(tv);
            b.s("    cvt.rn.f64.").s(op).c(' ').s(tr).s(", ").s(reg(o)).c(';');
        } else if (op && cstr_eq(op, "f32") && cstr_eq(fty, "f64")) {
            Str tr = reg(tv);
            b.s("    cvt.f64.f32 ").s(tr).s(", ").s(reg(o)).c(';');
        } else {
            return reg(o);
        }
        put(b);
        return reg(tv);
    }
    OCB_HD Str coerce_to_int(Opnd o, const char *ity) {
        if (o.k == O_CONST) return opnd(o, ity);
        if (o.k != O_VAL) { unsup(); return S("?"); }
        if (is_pred(vid(o))) return pred_to_int(o, ity);
        Ty t = V(o.x).ty;
        const char *op = is_ptr(t) ? nullptr : ptx_type(t);
        if (op && cstr_eq(op, ity)) return reg(o);
        const char *ints = " s8 u8 s16 u16 s32 u32 s64 u64 ";
        if (op && cstr_in(op, ints) && cstr_in(ity, ints)) {
            Ty mt = cstr_eq(ity, "s8") ? S_INT8 : cstr_eq(ity, "u8") ? S_UINT8 :
                    cstr_eq(ity, "s16") ? S_INT16 : cstr_eq(ity, "u16") ? S_UINT16 :
                    cstr_eq(ity, "s32") ? S_INT32 : cstr_eq(ity, "u32") ? S_UINT32 :
                    cstr_eq(ity, "s64") ? S_INT64 : S_UINT64;
            uint32_t tv = new_value(nm("_coerce_", vid(o)), mt);
            SB b = sb();
            Str tr = reg(tv);
            b.s("    cvt.").s(ity).c('.').s(op).c(' ').s(tr).s(", ").s(reg(o)).c(';');
            put(b);
            return reg(tv);
        }
        return reg(o);
    }
    // widen a 32-bit value through the kernel's widen cache
    OCB_HD int32_t widen_get(uint32_t id) { return id < widen_cap ? widen[id] : -1; }
    OCB_HD void widen_set(uint32_t id, uint32_t vx) {
        if (!grow_arr(widen, widen_cap, id, (int32_t)-1)) { unsup(); return; }
        widen[id] = (int32_t)vx;
    }

    // ---- _build_alloc_map (emit.py:115-342) ----------------------------------
    OCB_HD void build_alloc() {
        uint32_t n = nid0;
        alloc = (int32_t *)tmp.alloc(4ull * (n + 1), 16);
        Ty *vty = (Ty *)tmp.alloc(4ull * (n + 1), 16);
        int64_t *ls = (int64_t *)tmp.alloc(8ull * (n + 1), 16);
        int64_t *le = (int64_t *)tmp.alloc(8ull * (n + 1), 16);
        uint8_t *seen = (uint8_t *)tmp.alloc(n + 1, 16);
        uint32_t *order = (uint32_t *)tmp.alloc(4ull * (n + 1), 16);
        pred = (uint8_t *)tmp.alloc(n + 1, 16);
        pred_cap = n + 1;
        if (!alloc || !vty || !ls || !le || !seen || !order || !pred) { unsup(); return; }
        uint32_t no = 0;
        for (uint32_t i = 0; i <= n; ++i) {
            alloc[i] = -1;
            seen[i] = 0;
            pred[i] = 0;
        }
        auto note = [&](uint32_t id, Ty t, int64_t idx, bool def) {
            if (id >= n) { unsup(); return; }
            if (!seen[id]) {
                seen[id] = 1;
                order[no++] = id;
                vty[id] = t;
                ls[id] = idx;
                le[id] = idx;
                return;
            }
            if (def) {
                vty[id] = t;
                le[id] = idx;
            } else {
                if (idx < ls[id]) ls[id] = idx;
                if (idx > le[id]) le[id] = idx;
            }
        };
        auto def = [&](int32_t vx, int64_t idx) {
            if (vx >= 0) note(m.vals[vx].id, m.vals[vx].ty, idx, true);
        };
        auto use = [&](Opnd o, int64_t idx) {
            if (o.k == O_VAL) note(vid(o), V(o.x).ty, idx, false);
        };
        for (uint32_t i = 0; i < k->locals.n; ++i) def((int32_t)k->locals[i].val, 0);
        if (k->shared.n) {
            for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
                Block &b = B(k->blocks[bi]);
                for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                    const Inst &in = I(b.insts[ii]);
                    // getattr(inst, 'lhs'/'dest'/'addr'): BinInst/CmpInst have lhs;
                    // Load/Store have addr; every inst but Store has dest
                    Opnd cand[3];
                    int nc = 0;
                    if (in.kind == I_BIN || in.kind == I_CMP) cand[nc++] = in.a;
                    if (in.dest >= 0) cand[nc++] = ov((uint32_t)in.dest);
                    if (in.kind == I_LOAD || in.kind == I_STORE) cand[nc++] = in.a;
                    for (int q = 0; q < nc; ++q) {
                        if (cand[q].k != O_VAL) continue;
                        const Value &v = V(cand[q].x);
                        if (!is_ptr(v.ty)) continue;
                        bool sm = false;
                        for (uint32_t s = 0; s < k->shared.n && !sm; ++s) sm = eq(k->shared[s].name, v.name);
                        if (sm) def((int32_t)cand[q].x, 0);
                    }
                }
            }
        }
        // flat walk: instructions then the terminator of each block
        int64_t idx = 0;
        uint32_t nb = k->blocks.n;
        int64_t *bstart = (int64_t *)tmp.alloc(8ull * (nb + 1), 16);
        int64_t *bend = (int64_t *)tmp.alloc(8ull * (nb + 1), 16);
        if (!bstart || !bend) { unsup(); return; }
        for (uint32_t bi = 0; bi < nb; ++bi) {
            Block &b = B(k->blocks[bi]);
            bstart[bi] = idx;
            for (uint32_t ii = 0; ii < b.insts.n; ++ii, ++idx) {
                const Inst &in = I(b.insts[ii]);
                switch (in.kind) {
                case I_BIN:
                case I_CMP:
                case I_CVT:
                case I_SELECT:
                    def(in.dest, idx);
                    if (in.kind == I_CMP) add_pred(m.vals[in.dest].id);
                    break;
                default: break;
                }
                if (in.kind == I_BIN && (in.op == BO_AND || in.op == BO_OR || in.op == BO_XOR) &&
                    in.a.k == O_VAL && is_pred(vid(in.a)) && in.b.k == O_VAL && is_pred(vid(in.b)))
                    add_pred(m.vals[in.dest].id);
                if (in.kind == I_LOAD || in.kind == I_PARAM || in.kind == I_GADDR) def(in.dest, idx);
                if (in.kind == I_CALL && in.dest >= 0) def(in.dest, idx);
                switch (in.kind) {
                case I_BIN:
                case I_CMP:
                case I_STORE:
                    use(in.a, idx);
                    use(in.b, idx);
                    break;
                case I_SELECT:
                    use(in.c, idx);
                    use(in.a, idx);
                    use(in.b, idx);
                    break;
                case I_LOAD:
                case I_CVT: use(in.a, idx); break;
                case I_CALL:
                    for (uint32_t q = 0; q < in.args.n; ++q) use(in.args[q], idx);
                    if (in.dest >= 0) def(in.dest, idx);
                    break;
                case I_PRINTF:
                    for (uint32_t q = 0; q < in.args.n; ++q) use(in.args[q], idx);
                    break;
                case I_ASM:  // inputs used, then outputs defined (emit.py:225-231)
                    for (uint32_t q = in.pidx; q < in.args.n; ++q) use(in.args[q], idx);
                    for (uint32_t q = 0; q < in.pidx; ++q)
                        if (in.args[q].k == O_VAL) def((int32_t)in.args[q].x, idx);
                    break;
                default: break;
                }
            }
            if (b.term.kind != T_NONE) {
                if (b.term.kind == T_CBR || b.term.kind == T_RET) use(b.term.v, idx);
                ++idx;
            }
            bend[bi] = idx - 1;
        }
        if (bad()) return;
        // flat start/end per label (last block with a label wins)
        LabelMap lm;
        lm.build(tmp, m, k->blocks);
        IdArr<uint32_t> ordm;
        ordm.init(tmp, m.blocks.n, 0);
        for (uint32_t i = 0; i < nb; ++i) ordm.set(k->blocks[i], i);
        auto lab_ord = [&](Str l) -> int32_t {
            int32_t b = lm.get(l);
            return b < 0 ? -1 : (int32_t)ordm.get((uint32_t)b);
        };
        struct BE { int64_t hs, he, le; };
        Vec<BE> back;
        back.init();
        for (uint32_t bi = 0; bi < nb; ++bi) {
            Block &b = B(k->blocks[bi]);
            if (b.term.kind == T_NONE) continue;
            int32_t so = lab_ord(b.label);
            int64_t src_start = bstart[so];
            Str tg[2];
            int nt = 0;
            if (b.term.kind == T_BR) tg[nt++] = b.term.t;
            else if (b.term.kind == T_CBR) { tg[nt++] = b.term.t; tg[nt++] = b.term.f; }
            for (int q = 0; q < nt; ++q) {
                int32_t to = lab_ord(tg[q]);
                if (to >= 0 && bstart[to] <= src_start) back.push(tmp, BE{bstart[to], bend[to], bend[so]});
            }
        }
        for (uint32_t e = 0; e < back.n; ++e) {
            for (uint32_t q = 0; q < no; ++q) {
                uint32_t id = order[q];
                int64_t lend = le[id], lstart = ls[id];
                if (!(back[e].hs <= lend && lend <= back[e].le)) continue;
                bool classic = lstart <= back[e].hs;
                bool inline_merge = lstart <= back[e].he && lend > back[e].he;
                if (classic || inline_merge) le[id] = back[e].le;
            }
        }
        // linear scan per prefix bucket
        for (int pf = 0; pf < PF_N; ++pf) alloc_max[pf] = 0;
        for (int pf = 0; pf < PF_N; ++pf) {
            uint32_t cnt = 0;
            for (uint32_t q = 0; q < no; ++q) {
                uint32_t id = order[q];
                int p = is_pred(id) ? PF_P : reg_prefix(vty[id]);
                if (p == pf) cnt++;
            }
            if (!cnt) continue;
            struct Iv { int64_t s, e; uint32_t id; };
            Iv *iv = (Iv *)tmp.alloc(sizeof(Iv) * (uint64_t)cnt, 16);
            Iv *act = (Iv *)tmp.alloc(sizeof(Iv) * (uint64_t)cnt, 16);
            int32_t *act_phys = (int32_t *)tmp.alloc(4ull * cnt, 16);
            int32_t *freel = (int32_t *)tmp.alloc(4ull * (cnt + 1), 16);
            if (!iv || !act || !act_phys || !freel) { unsup(); return; }
            uint32_t c2 = 0;
            for (uint32_t q = 0; q < no; ++q) {
                uint32_t id = order[q];
                int p = is_pred(id) ? PF_P : reg_prefix(vty[id]);
                if (p == pf) iv[c2++] = Iv{ls[id], le[id], id};
            }
            // stable sort by start (insertion sort on runs is fine here)
            for (uint32_t a = 1; a < cnt; ++a) {
                Iv x = iv[a];
                int32_t j = (int32_t)a - 1;
                while (j >= 0 && iv[j].s > x.s) {
                    iv[j + 1] = iv[j];
                    --j;
                }
                iv[j + 1] = x;
            }
            uint32_t nact = 0, fhead = 0, ftail = 0;
            int next_reg = 0;
            bool reuse = pf != PF_R;
            for (uint32_t q = 0; q < cnt; ++q) {
                uint32_t w = 0;
                for (uint32_t a = 0; a < nact; ++a) {
                    if (act[a].e < iv[q].s) {
                        if (reuse) freel[ftail++] = act_phys[a];
                    } else {
                        act[w] = act[a];
                        act_phys[w] = act_phys[a];
                        ++w;
                    }
                }
                nact = w;
                int phys;
                if (fhead < ftail) phys = freel[fhead++];
                else phys = next_reg++;
                alloc[iv[q].id] = phys;
                act[nact] = iv[q];
                act_phys[nact] = phys;
                ++nact;
                if (alloc_max[pf] < phys + 1) alloc_max[pf] = phys + 1;
            }
        }
    }

    // ---- declared here, defined in cc_emit_inst.cuh ------------------------
    OCB_HD OCB_NI void emit_inst(uint32_t ix);
    OCB_HD OCB_NI void emit_bin(const Inst &in);
    OCB_HD OCB_NI void emit_cmp(const Inst &in);
    OCB_HD OCB_NI void emit_cvt(const Inst &in);
    OCB_HD OCB_NI void emit_load(const Inst &in);
    OCB_HD OCB_NI void emit_store(const Inst &in);
    OCB_HD OCB_NI void emit_call(const Inst &in);
    OCB_HD OCB_NI void emit_printf(const Inst &in);
    OCB_HD OCB_NI void emit_asm(const Inst &in);
    OCB_HD OCB_NI void emit_math(const Inst &in, Str dest);
    OCB_HD OCB_NI void emit_term(const Term &t);
    OCB_HD OCB_NI void emit_block(uint32_t b);
    OCB_HD OCB_NI void peepholes(Vec<Str> &body);
    OCB_HD OCB_NI bool rd_compact(Vec<Str> &L);
    OCB_HD OCB_NI bool emit_devfn(Kernel &f, Vec<Str> &out);
    OCB_HD OCB_NI bool emit_kernel(Kernel &kk, Vec<Str> &out);
    OCB_HD int32_t block_by_label(Str l);
    OCB_HD OCB_NI LblEnt *label_slot(Str l, bool create);
    OCB_HD uint32_t pred_count_of(Str l);
};

}  // namespace cc
}  // namespace ocb
