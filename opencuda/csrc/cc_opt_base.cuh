// Optimizer building blocks shared with the emitter: Python value semantics
// of IR constants, id-indexed scratch arrays, label maps and sets, and the
// keys and per-block tables of CSE (opencuda/ir/optimize.py:397-640).
#pragma once
#include "cc_ir.cuh"

namespace ocb {
namespace cc {

// ---------------------------------------------------------------------------
// Python value helpers for Const
// ---------------------------------------------------------------------------
struct PyVal {
    uint8_t isf;  // 1 = float
    pyint i;
    double f;
};
OCB_HD inline PyVal pv_int(pyint i) { return PyVal{0, i, 0.0}; }
OCB_HD inline PyVal pv_float(double f) { return PyVal{1, 0, f}; }
OCB_HD inline PyVal pv_of(const Const &c) { return PyVal{c.pyfloat, c.i, c.f}; }
OCB_HD inline bool is_finite(double f) { return f == f && f - f == 0.0; }

// exact comparison of an int with a float (Python int/float ordering)
// returns -1, 0, 1; 2 when b is NaN (unordered)
OCB_HD inline int cmp_int_float(pyint a, double b) {
    if (b != b) return 2;
    if (b >= 1.7e38) return -1;   // beyond any kept pyint
    if (b <= -1.7e38) return 1;
    double fb = floor(b);
    pyint ib = (pyint)fb;
    if (a < ib) return -1;
    if (a > ib) return 1;
    return b == fb ? 0 : -1;
}
// Python ==
OCB_HD inline bool pv_eq(const PyVal &a, const PyVal &b) {
    if (!a.isf && !b.isf) return a.i == b.i;
    if (a.isf && b.isf) return a.f == b.f;
    if (a.isf) return cmp_int_float(b.i, a.f) == 0;
    return cmp_int_float(a.i, b.f) == 0;
}
// Python a > b (False when unordered)
OCB_HD inline bool pv_gt(const PyVal &a, const PyVal &b) {
    if (!a.isf && !b.isf) return a.i > b.i;
    if (a.isf && b.isf) return a.f > b.f;
    if (a.isf) {
        int c = cmp_int_float(b.i, a.f);
        return c == -1;
    }
    int c = cmp_int_float(a.i, b.f);
    return c == 1;
}
OCB_HD inline bool pv_eq_int(const PyVal &a, pyint v) { return pv_eq(a, pv_int(v)); }
OCB_HD inline bool pv_truthy(const PyVal &a) { return a.isf ? a.f != 0.0 : a.i != 0; }
// int(value): false when Python raises (NaN/inf) or leaves the kept range
OCB_HD inline bool pv_to_int(const PyVal &a, pyint &out) {
    if (!a.isf) {
        out = a.i;
        return true;
    }
    if (!is_finite(a.f) || a.f >= 1.3e36 || a.f <= -1.3e36) return false;
    out = (pyint)trunc(a.f);
    return true;
}
OCB_HD inline double pv_to_float(const PyVal &a) { return a.isf ? a.f : (double)a.i; }

// Python float % (CPython float_rem: fmod, then the sign of the divisor)
OCB_HD inline double py_fmod(double vx, double wx) {
    double mod = fmod(vx, wx);
    if (mod != 0.0) {
        if ((wx < 0) != (mod < 0)) mod += wx;
    } else {
        mod = copysign(0.0, wx);
    }
    return mod;
}

// _mask_int (optimize.py:53-70): wrap to the type's width with its sign.
// `ok` is false where the reference would keep an unbounded value we cannot.
OCB_HD inline pyint mask_int_wrapped(pyint wrapped_low, Ty ty) {
    uint32_t bits = ty_size(ty) * 8;
    unsigned __int128 mask = bits >= 128 ? ~(unsigned __int128)0
                                         : (((unsigned __int128)1) << bits) - 1;
    unsigned __int128 v = (unsigned __int128)wrapped_low & mask;
    if (ty_is_signed(ty) && bits && ((v >> (bits - 1)) & 1)) {
        return (pyint)v - (pyint)(((unsigned __int128)1) << bits);
    }
    return (pyint)v;
}
OCB_HD inline bool masks(Ty ty) { return !is_ptr(ty) && !ty_is_float(ty); }

// ---------------------------------------------------------------------------
// per-pass scratch: id-indexed arrays and a label -> block map
// ---------------------------------------------------------------------------
template <class T>
struct IdArr {
    T *p;
    uint32_t n;
    T dflt;
    OCB_HD void init(Arena &a, uint32_t size, T d) {
        n = size;
        dflt = d;
        p = (T *)a.alloc(sizeof(T) * (uint64_t)(size ? size : 1), 16);
        if (p)
            for (uint32_t i = 0; i < size; ++i) p[i] = d;
        else
            n = 0;
    }
    OCB_HD T get(uint32_t id) const { return id < n ? p[id] : dflt; }
    OCB_HD bool set(uint32_t id, T v) {
        if (id >= n) return false;
        p[id] = v;
        return true;
    }
};

struct LabelMap {
    int32_t *ht;
    uint32_t cap;
    const Module *m;
    OCB_HD void build(Arena &a, const Module &mod, const Vec<uint32_t> &blocks) {
        m = &mod;
        cap = 16;
        while (cap < 2 * blocks.n + 2) cap *= 2;
        ht = (int32_t *)a.alloc(4ull * cap, 16);
        if (!ht) {
            cap = 0;
            return;
        }
        for (uint32_t i = 0; i < cap; ++i) ht[i] = -1;
        for (uint32_t i = 0; i < blocks.n; ++i) put(blocks[i]);
    }
    OCB_HD void put(uint32_t b) {  // last wins, like a dict comprehension
        Str l = m->blocks[b].label;
        uint32_t h = hash(l) & (cap - 1);
        while (ht[h] >= 0) {
            if (eq(m->blocks[ht[h]].label, l)) {
                ht[h] = (int32_t)b;
                return;
            }
            h = (h + 1) & (cap - 1);
        }
        ht[h] = (int32_t)b;
    }
    OCB_HD int32_t get(Str l) const {
        if (!cap) return -1;
        uint32_t h = hash(l) & (cap - 1);
        while (ht[h] >= 0) {
            if (eq(m->blocks[ht[h]].label, l)) return ht[h];
            h = (h + 1) & (cap - 1);
        }
        return -1;
    }
};

// A set of labels (open addressing over Str).
struct LabelSet {
    Str *ht;
    uint32_t cap, n;
    OCB_HD void init(Arena &a, uint32_t want) {
        cap = 16;
        while (cap < 2 * want + 2) cap *= 2;
        n = 0;
        ht = (Str *)a.alloc(sizeof(Str) * (uint64_t)cap, 16);
        if (!ht) {
            cap = 0;
            return;
        }
        for (uint32_t i = 0; i < cap; ++i) ht[i] = Str{nullptr, 0};
    }
    OCB_HD bool has(Str l) const {
        if (!cap) return false;
        uint32_t h = hash(l) & (cap - 1);
        while (ht[h].p) {
            if (eq(ht[h], l)) return true;
            h = (h + 1) & (cap - 1);
        }
        return false;
    }
    OCB_HD bool add(Str l) {  // true when newly added
        if (!cap) return false;
        uint32_t h = hash(l) & (cap - 1);
        while (ht[h].p) {
            if (eq(ht[h], l)) return false;
            h = (h + 1) & (cap - 1);
        }
        if (2 * (n + 1) > cap) return false;  // sized by the caller
        ht[h] = l;
        ++n;
        return true;
    }
};

// CSE keys (optimize.py:397-640).  An operand key is the reference's tuple
// ('val', id) or ('const', value); here the constant is kept as its index in
// the TU's constant pool and compared by Python value through the pool (so
// 1 == 1.0 as there), which keeps a key at 8 bytes and a table entry at 28.
struct OKey {
    uint8_t tag;  // 0 'const' (x = constant index), 1 'val' (x = value id)
    uint32_t x;
};
struct CKey {
    uint8_t kind;  // 0 bin, 1 cvt, 2 cmp, 3 pure call
    uint8_t op;    // bin/cmp operator; pure call: builtin code
    OKey l, r;
    uint32_t t1, t2;  // str(type) keys
};
OCB_HD inline bool okey_eq(const OKey &a, const OKey &b, const Const *cs) {
    if (a.tag != b.tag) return false;
    if (a.tag == 1 || a.x == b.x) return a.x == b.x;
    return pv_eq(pv_of(cs[a.x]), pv_of(cs[b.x]));
}
// tuple a > tuple b for ('const', v) / ('val', id)
OCB_HD inline bool okey_gt(const OKey &a, const OKey &b, const Const *cs) {
    if (a.tag != b.tag) return a.tag > b.tag;
    if (a.tag == 1) return a.x > b.x;
    PyVal va = pv_of(cs[a.x]), vb = pv_of(cs[b.x]);
    if (pv_eq(va, vb)) return false;
    return pv_gt(va, vb);
}
OCB_HD inline uint32_t okey_hash(const OKey &k, const Const *cs) {
    if (k.tag == 1) return k.x * 2654435761u + 7;
    // numeric hash: integral floats hash like ints
    const Const &c = cs[k.x];
    pyint iv;
    if (c.pyfloat) {
        double f = c.f;
        if (is_finite(f) && f == trunc(f) && f < 1e30 && f > -1e30) iv = (pyint)f;
        else {
            uint64_t b;
            memcpy(&b, &f, 8);
            return (uint32_t)(b ^ (b >> 29)) * 0x9E3779B1u;
        }
    } else {
        iv = c.i;
    }
    uint64_t lo = (uint64_t)iv, hi = (uint64_t)((unsigned __int128)iv >> 64);
    return (uint32_t)((lo ^ (lo >> 31) ^ (hi * 31)) * 0x9E3779B1u);
}
OCB_HD inline bool ckey_eq(const CKey &a, const CKey &b, const Const *cs) {
    if (a.kind != b.kind) return false;
    if (a.kind == 3) return a.op == b.op;
    if (a.kind != 1 && a.op != b.op) return false;
    if (!okey_eq(a.l, b.l, cs)) return false;
    if (a.kind == 1) return a.t1 == b.t1 && a.t2 == b.t2;
    if (!okey_eq(a.r, b.r, cs)) return false;
    return a.kind == 2 || a.t1 == b.t1;
}
OCB_HD inline uint32_t ckey_hash(const CKey &k, const Const *cs) {
    if (k.kind == 3) return k.op * 0x9E3779B1u ^ 0x55u;
    uint32_t h = k.kind * 31u + (k.kind == 1 ? 0 : k.op);
    h = h * 1000003u ^ okey_hash(k.l, cs);
    if (k.kind != 1) h = h * 1000003u ^ okey_hash(k.r, cs);
    if (k.kind != 2) h = h * 1000003u ^ k.t1;
    if (k.kind == 1) h = h * 1000003u ^ k.t2;
    return h;
}

// The `seen` dict of one block: key -> value index.
struct Seen {
    struct E {
        CKey k;
        uint32_t v;
        uint32_t used;
    };
    E *t;
    uint32_t cap, n;
    const Const *cs;  // the TU's constant pool (keys hold indices into it)
    OCB_HD bool init(Arena &a, uint32_t c, const Const *consts) {
        cs = consts;
        cap = 16;
        while (cap < c) cap *= 2;
        n = 0;
        t = (E *)a.alloc(sizeof(E) * (uint64_t)cap, 16);
        if (!t) return false;
        for (uint32_t i = 0; i < cap; ++i) t[i].used = 0;
        return true;
    }
    OCB_HD int32_t find(const CKey &k) const {
        uint32_t h = ckey_hash(k, cs) & (cap - 1);
        while (t[h].used) {
            if (ckey_eq(t[h].k, k, cs)) return (int32_t)t[h].v;
            h = (h + 1) & (cap - 1);
        }
        return -1;
    }
    OCB_HD bool grow(Arena &a) {
        Seen s2;
        if (!s2.init(a, cap * 2, cs)) return false;
        for (uint32_t i = 0; i < cap; ++i)
            if (t[i].used) s2.put_new(t[i].k, t[i].v);
        *this = s2;
        return true;
    }
    OCB_HD void put_new(const CKey &k, uint32_t v) {
        uint32_t h = ckey_hash(k, cs) & (cap - 1);
        while (t[h].used) {
            if (ckey_eq(t[h].k, k, cs)) {
                t[h].v = v;
                return;
            }
            h = (h + 1) & (cap - 1);
        }
        t[h].k = k;
        t[h].v = v;
        t[h].used = 1;
        n++;
    }
    OCB_HD bool put(Arena &a, const CKey &k, uint32_t v) {
        if (2 * (n + 1) > cap && !grow(a)) return false;
        put_new(k, v);
        return true;
    }
    OCB_HD bool copy_from(Arena &a, const Seen &o) {
        cs = o.cs;
        cap = o.cap;
        n = o.n;
        t = (E *)a.alloc(sizeof(E) * (uint64_t)cap, 16);
        if (!t) return false;
        for (uint32_t i = 0; i < cap; ++i) t[i] = o.t[i];
        return true;
    }
};

}  // namespace cc
}  // namespace ocb
