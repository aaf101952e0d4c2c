// Compiler core data model (host+device C++): per-TU arena, strings, types,
// and the SSA IR of opencuda/ir/nodes.py:23-289 / ir/types.py:15-142.
//
// One thread compiles one TU inside a private arena of global memory; every
// container grows inside that arena (nothing is freed until the TU is done).
// Running out of arena sets `oom`, which the driver reports as
// OCB_TU_OVERFLOW and retries with a larger arena.
#pragma once
#include <stdint.h>
#include <string.h>

#ifndef OCB_HD
#define OCB_HD __host__ __device__
#endif
// Large or recursive routines stay out of line: inlining them all into one
// kernel only grows compile time and register pressure.
#ifndef OCB_NI
#ifdef __CUDACC__
#define OCB_NI __noinline__
#else
#define OCB_NI __attribute__((noinline))
#endif
#endif

namespace ocb {
namespace cc {

// ---------------------------------------------------------------------------
// Python int values of constants: 128-bit, kept inside +-2^120 (a TU whose
// constant arithmetic leaves that range is outside the subset)
// ---------------------------------------------------------------------------
typedef __int128 pyint;
#define PYINT_LIM (((pyint)1) << 120)
OCB_HD inline bool py_ok(pyint v) { return v < PYINT_LIM && v > -PYINT_LIM; }
OCB_HD inline pyint py_abs(pyint v) { return v < 0 ? -v : v; }
// a * b, false when the product leaves the range
OCB_HD inline bool py_mul(pyint a, pyint b, pyint &r) {
    if (a == 0 || b == 0) {
        r = 0;
        return true;
    }
    if (py_abs(a) > PYINT_LIM / py_abs(b)) return false;
    r = a * b;
    return py_ok(r);
}
// number of bits of |v| (int.bit_length)
OCB_HD inline int py_bitlen(pyint v) {
    unsigned __int128 u = (unsigned __int128)py_abs(v);
    int n = 0;
    while (u) {
        u >>= 1;
        ++n;
    }
    return n;
}
// a << s for s >= 0
OCB_HD inline bool py_shl(pyint a, pyint s, pyint &r) {
    if (a == 0) {
        r = 0;
        return true;
    }
    if (s < 0 || s > 120 || py_bitlen(a) + (int)s >= 120) return false;
    r = a * (((pyint)1) << (int)s);
    return true;
}
// a >> s for s >= 0 (floor semantics, like Python)
OCB_HD inline pyint py_shr(pyint a, pyint s) {
    if (s >= 127) return a < 0 ? -1 : 0;
    int k = (int)s;
    // written with unsigned shifts: floor(a / 2^k) for both signs
    if (a >= 0) return (pyint)((unsigned __int128)a >> k);
    return ~(pyint)((unsigned __int128)~a >> k);
}

// ---------------------------------------------------------------------------
// arena + growable vectors
// ---------------------------------------------------------------------------
// A TU's slice is a bump allocator.  When an allocation does not fit, it is
// taken from the launch's shared spill pool (one atomic add; spilled blocks
// are never reused, resets of `used` only rewind the slice); `oom` is set
// only when the pool is exhausted too, and the driver then reruns the TU
// with a larger slice.
struct SpillPool {
    uint8_t *base;
    unsigned long long *top;   // bytes handed out so far (device counter)
    uint64_t cap;
};

struct Arena {
    uint8_t *base;
    uint64_t used, cap;
    bool oom;
    SpillPool spill = {nullptr, nullptr, 0};
    OCB_HD void *spill_alloc(uint64_t n, uint64_t align) {
        if (!spill.top) return nullptr;
        uint64_t want = (n + align + 15) & ~15ull;
#ifdef __CUDA_ARCH__
        uint64_t o = atomicAdd(spill.top, (unsigned long long)want);
#else
        uint64_t o = *spill.top;
        *spill.top += want;
#endif
        if (o + want > spill.cap) return nullptr;
        uintptr_t p = ((uintptr_t)(spill.base + o) + align - 1) & ~(uintptr_t)(align - 1);
        return (void *)p;
    }
    OCB_HD void *alloc(uint64_t n, uint64_t align = 8) {
        uint64_t a = (used + align - 1) & ~(align - 1);
        if (a + n > cap) {
            void *p = spill_alloc(n, align);
            if (!p) oom = true;
            return p;
        }
        used = a + n;
#ifdef OCB_ARENA_PEAK
        if (used > peak) peak = used;
#endif
        return base + a;
    }
#ifdef OCB_ARENA_PEAK
    uint64_t peak = 0;
#endif
};

template <class T>
struct Vec {
    T *p;
    uint32_t n, cap;
    OCB_HD void init() { p = nullptr; n = cap = 0; }
    OCB_HD bool reserve(Arena &a, uint32_t want) {
        if (want <= cap) return true;
        uint32_t nc = cap ? cap * 2 : 8;
        while (nc < want) nc *= 2;
        T *np = (T *)a.alloc(sizeof(T) * (uint64_t)nc, alignof(T) < 8 ? 8 : alignof(T));
        if (!np) return false;
        for (uint32_t i = 0; i < n; ++i) np[i] = p[i];
        p = np;
        cap = nc;
        return true;
    }
    OCB_HD bool push(Arena &a, const T &v) {
        if (n == cap && !reserve(a, n + 1)) return false;
        p[n++] = v;
        return true;
    }
    OCB_HD T &operator[](uint32_t i) { return p[i]; }
    OCB_HD const T &operator[](uint32_t i) const { return p[i]; }
    OCB_HD T &back() { return p[n - 1]; }
    OCB_HD void erase(uint32_t i) {
        for (uint32_t k = i + 1; k < n; ++k) p[k - 1] = p[k];
        --n;
    }
    OCB_HD bool insert(Arena &a, uint32_t i, const T &v) {
        if (n == cap && !reserve(a, n + 1)) return false;
        for (uint32_t k = n; k > i; --k) p[k] = p[k - 1];
        p[i] = v;
        ++n;
        return true;
    }
    OCB_HD Vec copy(Arena &a) const {
        Vec r;
        r.init();
        if (n && r.reserve(a, n)) {
            for (uint32_t i = 0; i < n; ++i) r.p[i] = p[i];
            r.n = n;
        }
        return r;
    }
};

// ---------------------------------------------------------------------------
// strings (not NUL terminated)
// ---------------------------------------------------------------------------
struct Str {
    const char *p;
    uint32_t n;
};
OCB_HD inline uint32_t cstrlen(const char *s) {
    uint32_t n = 0;
    while (s[n]) ++n;
    return n;
}
OCB_HD inline Str S(const char *s) { return Str{s, cstrlen(s)}; }
OCB_HD inline bool eq(Str a, Str b) {
    if (a.n != b.n) return false;
    for (uint32_t i = 0; i < a.n; ++i)
        if (a.p[i] != b.p[i]) return false;
    return true;
}
OCB_HD inline bool eq(Str a, const char *b) {
    uint32_t i = 0;
    for (; i < a.n; ++i)
        if (b[i] != a.p[i] || !b[i]) return false;
    return b[i] == 0;
}
OCB_HD inline bool mem_eq(const char *a, const char *b, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i)
        if (a[i] != b[i]) return false;
    return true;
}
OCB_HD inline bool starts(Str a, const char *b) {
    uint32_t i = 0;
    for (; b[i]; ++i)
        if (i >= a.n || a.p[i] != b[i]) return false;
    return true;
}
OCB_HD inline bool ends_with(Str a, const char *b) {
    uint32_t n = 0;
    while (b[n]) ++n;
    return n <= a.n && mem_eq(a.p + a.n - n, b, n);
}
OCB_HD inline uint32_t hash(Str s) {
    uint32_t h = 2166136261u;
    for (uint32_t i = 0; i < s.n; ++i) h = (h ^ (uint8_t)s.p[i]) * 16777619u;
    return h;
}
// a ++ b (++ c)
OCB_HD inline Str cat(Arena &a, Str x, Str y, Str z = Str{nullptr, 0}) {
    char *d = (char *)a.alloc(x.n + y.n + z.n + 1, 1);
    if (!d) return Str{"?", 1};
    uint32_t k = 0;
    for (uint32_t i = 0; i < x.n; ++i) d[k++] = x.p[i];
    for (uint32_t i = 0; i < y.n; ++i) d[k++] = y.p[i];
    for (uint32_t i = 0; i < z.n; ++i) d[k++] = z.p[i];
    d[k] = 0;
    return Str{d, k};
}
OCB_HD inline Str utoa(Arena &a, uint64_t v) {
    char tmp[24];
    int k = 0;
    do {
        tmp[k++] = (char)('0' + v % 10);
        v /= 10;
    } while (v);
    char *d = (char *)a.alloc(k + 1, 1);
    if (!d) return Str{"0", 1};
    for (int i = 0; i < k; ++i) d[i] = tmp[k - 1 - i];
    d[k] = 0;
    return Str{d, (uint32_t)k};
}

// ---------------------------------------------------------------------------
// types (ir/types.py): packed so that == is the reference's structural ==
//   bits 0-3 scalar, 4-5 pointer depth, 6-8 outer address space,
//   9 volatile of the innermost pointer, 10 volatile of the outer pointer,
//   16-31 the struct index of a StructTy (scalar code S_STRUCT)
// ---------------------------------------------------------------------------
typedef uint32_t Ty;
enum : uint32_t {
    S_VOID = 0, S_BOOL, S_INT8, S_UINT8, S_INT16, S_UINT16, S_INT32, S_UINT32,
    S_INT64, S_UINT64, S_FLOAT, S_DOUBLE, S_HALF,
    S_STRUCT  // StructTy (ir/types.py:107-142): bits 16-31 index Module::structs
};
// AS_INT0: the integer 0 the reference stores as the space of an array
// parameter's pointer (PtrTy(ty, 0)); it is none of the named spaces.
enum : uint32_t { AS_GENERIC = 0, AS_GLOBAL, AS_SHARED, AS_LOCAL, AS_CONST, AS_INT0 };

OCB_HD inline Ty ty_s(uint32_t s) { return s; }
OCB_HD inline uint32_t ty_depth(Ty t) { return (t >> 4) & 3; }
OCB_HD inline bool is_ptr(Ty t) { return ty_depth(t) != 0; }
OCB_HD inline uint32_t ty_scalar(Ty t) { return t & 15; }
OCB_HD inline uint32_t ty_as(Ty t) { return (t >> 6) & 7; }
OCB_HD inline bool ty_vol(Ty t) {  // PtrTy.volatile of the outermost pointer
    return ty_depth(t) == 1 ? ((t >> 9) & 1) : ((t >> 10) & 1);
}
// PtrTy(pointee, as, vol), up to three levels; representable when only the
// outermost pointer has a non-global address space and volatile sits on the
// innermost or outermost one.
OCB_HD inline Ty ty_ptr(Ty pointee, uint32_t as, bool vol, bool &ok) {
    uint32_t d = ty_depth(pointee);
    if (d == 0) return pointee | (1u << 4) | (as << 6) | (vol ? 1u << 9 : 0);
    if (d >= 3 || ty_as(pointee) != AS_GLOBAL || ((pointee >> 10) & 1)) {
        ok = false;
        return pointee;
    }
    return (pointee & ~((3u << 4) | (7u << 6))) | ((d + 1) << 4) | (as << 6) | (vol ? 1u << 10 : 0);
}
OCB_HD inline Ty ty_pointee(Ty t) {
    uint32_t d = ty_depth(t);
    if (d <= 1) return t & (15u | 0xFFFF0000u);
    return (t & ~((3u << 4) | (7u << 6) | (1u << 10))) | ((d - 1) << 4) | (AS_GLOBAL << 6);
}
OCB_HD inline Ty ty_struct(uint32_t idx) { return S_STRUCT | (idx << 16); }
OCB_HD inline bool ty_is_struct(Ty t) { return !is_ptr(t) && (t & 15) == S_STRUCT; }
OCB_HD inline uint32_t ty_sidx(Ty t) { return t >> 16; }
// a ScalarTy (not a pointer, not a struct)
OCB_HD inline bool ty_is_scalar(Ty t) { return !is_ptr(t) && (t & 15) != S_STRUCT; }
// size of a scalar or pointer type (a struct's size is Module::tsize)
OCB_HD inline uint32_t ty_size(Ty t) {
    if (is_ptr(t)) return 8;
    switch (ty_scalar(t)) {
    case S_STRUCT: return 0;
    case S_VOID: return 0;
    case S_BOOL: case S_INT8: case S_UINT8: return 1;
    case S_INT16: case S_UINT16: case S_HALF: return 2;
    case S_INT32: case S_UINT32: case S_FLOAT: return 4;
    default: return 8;
    }
}
OCB_HD inline bool ty_is_float(Ty t) {
    uint32_t s = ty_scalar(t);
    return !is_ptr(t) && (s == S_FLOAT || s == S_DOUBLE || s == S_HALF);
}
OCB_HD inline bool ty_is_signed(Ty t) {
    uint32_t s = ty_scalar(t);
    return !is_ptr(t) && (s == S_INT8 || s == S_INT16 || s == S_INT32 || s == S_INT64);
}
// str(ty) equality key (ir/types.py __str__): pointers ignore address space
OCB_HD inline uint32_t ty_strkey(Ty t) { return is_ptr(t) ? (t & ~(7u << 6)) : t; }
OCB_HD inline const char *scalar_name(uint32_t s) {
    switch (s) {
    case S_VOID: return "void";
    case S_BOOL: return "bool";
    case S_INT8: return "char";
    case S_UINT8: return "unsigned char";
    case S_INT16: return "short";
    case S_UINT16: return "unsigned short";
    case S_INT32: return "int";
    case S_UINT32: return "unsigned int";
    case S_INT64: return "long long";
    case S_UINT64: return "unsigned long long";
    case S_FLOAT: return "float";
    case S_DOUBLE: return "double";
    default: return "half";
    }
}
OCB_HD inline const char *as_name(uint32_t a) {
    switch (a) {
    case AS_GENERIC: return "generic";
    case AS_GLOBAL: return "global";
    case AS_SHARED: return "shared";
    case AS_LOCAL: return "local";
    case AS_INT0: return "0";
    default: return "const";
    }
}

// ---------------------------------------------------------------------------
// IR
// ---------------------------------------------------------------------------
struct Value {
    uint32_t id;
    Ty ty;
    Str name;
};
struct Const {
    Ty ty;
    uint8_t pyfloat;  // the reference holds a Python float (else an int)
    pyint i;
    double f;
};
// O_SYM: a module-level __device__ / __constant__ symbol used directly as an
// address (the reference's SymbolRef); x indexes Module::gvars.
enum : uint8_t { O_NONE = 0, O_VAL = 1, O_CONST = 2, O_SYM = 3 };
struct Opnd {
    uint8_t k;
    uint32_t x;  // index into values / consts / gvars
};
OCB_HD inline Opnd ov(uint32_t v) { return Opnd{O_VAL, v}; }
OCB_HD inline Opnd oc(uint32_t c) { return Opnd{O_CONST, c}; }
OCB_HD inline Opnd onone() { return Opnd{O_NONE, 0}; }

enum : uint8_t { BO_ADD = 0, BO_SUB, BO_MUL, BO_DIV, BO_MOD, BO_AND, BO_OR, BO_XOR, BO_SHL, BO_SHR };
enum : uint8_t { CO_EQ = 0, CO_NE, CO_LT, CO_LE, CO_GT, CO_GE };
OCB_HD inline const char *binop_name(uint8_t o) {
    const char *n[] = {"add", "sub", "mul", "div", "mod", "and", "or", "xor", "shl", "shr"};
    return n[o];
}
OCB_HD inline const char *cmpop_name(uint8_t o) {
    const char *n[] = {"==", "!=", "<", "<=", ">", ">="};
    return n[o];
}

// I_GADDR: the address of a module symbol into a u64 register (GlobalAddrInst,
// ir/nodes.py:166-178); func = symbol name, op = its address space.
// I_PRINTF: printf(fmt, args...) (PrintfInst, ir/nodes.py:159-163); func =
// the format string with the parser's escapes resolved, args = the values.
// I_ASM: inline PTX (AsmInst, ir/nodes.py:180-189); func = the template,
// args = the output values then the input operands, pidx = output count.
enum : uint8_t { I_BIN = 0, I_CMP, I_SELECT, I_LOAD, I_STORE, I_CVT, I_CALL, I_PARAM, I_GADDR,
                 I_PRINTF, I_ASM };
struct Inst {
    uint8_t kind, op;
    int32_t dest;     // value index, -1 = none
    Opnd a, b, c;     // bin/cmp: a op b; select: c ? a : b; load: a; store: a <- b; cvt: a
    Str func;         // call: builtin name; param: name
    uint32_t pidx;    // param index
    Vec<Opnd> args;   // call arguments
};

enum : uint8_t { T_NONE = 0, T_RET, T_BR, T_CBR };
struct Term {
    uint8_t kind;
    Opnd v;           // ret value / branch condition
    Str t, f;         // targets
};

struct Block {
    Str label;
    Vec<uint32_t> insts;  // instruction indices
    Term term;
};

struct Param {
    Str name;
    Ty ty;
};
struct SharedDecl {
    Str name;
    Ty ty;
    int64_t count;
};
struct LocalDecl {
    Str name;
    Ty ty;
    int64_t count;
    uint32_t val;
};

struct Kernel {
    Str name;
    Vec<Param> params;
    Vec<uint32_t> blocks;     // block indices, in reference order
    uint32_t next_id;
    int64_t launch[2];
    uint8_t n_launch;
    Vec<SharedDecl> shared;
    Vec<LocalDecl> locals;
    bool has_locals;           // the reference created _local_decls
    Ty ret;                    // a device function's return type (S_VOID for kernels)
};

// A module-level variable (Module.global_vars, ir/nodes.py:289): element
// type, element count, address space (AS_GLOBAL or AS_CONST), and the
// pointer type its symbol carries.
struct GVar {
    Str name;
    Ty elem, ptr;
    uint32_t count;
    uint32_t space;
};

// A struct or union type (StructTy: name and ordered fields; a union is laid
// out as a struct, as there).  Array members `T a[N]` are N fields a_0..a_N-1.
struct SField {
    Str name;
    Ty ty;
};
struct StructDef {
    Str name;
    uint32_t f0, nf;  // fields: Module::sfields[f0, f0 + nf)
    uint32_t size;    // StructTy.size
};

// All IR objects of one TU.
struct Module {
    Arena *ar;
    Vec<Value> vals;
    Vec<Const> consts;
    Vec<Inst> insts;
    Vec<Block> blocks;
    Vec<Kernel> kernels;
    Vec<Kernel> funcs;        // recursive __device__ functions (DeviceFunction), .func
    Vec<GVar> gvars;          // in declaration order
    Vec<StructDef> structs;   // every StructTy of the TU (Ty bits 16-31 index it)
    Vec<SField> sfields;
    bool unsup;               // the engine cannot reproduce this TU
    int raises;               // reference exception (OCB_TU_RAISES_*) or 0

    OCB_HD void init(Arena *a) {
        ar = a;
        vals.init();
        consts.init();
        insts.init();
        blocks.init();
        kernels.init();
        funcs.init();
        gvars.init();
        structs.init();
        sfields.init();
        unsup = false;
        raises = 0;
        // Reserved up front so the tables are never empty-and-unallocated: a
        // push that fails later (arena exhausted, TU reported as OVERFLOW)
        // then returns an existing index instead of one past an empty table.
        vals.reserve(*a, 64);
        consts.reserve(*a, 64);
        insts.reserve(*a, 64);
        blocks.reserve(*a, 16);
        kernels.reserve(*a, 4);
    }
    // Type.size of any type (StructTy.size for structs, types.py:113-124:
    // each field aligned to its own size, no tail padding)
    OCB_HD uint32_t tsize(Ty t) const {
        if (ty_is_struct(t)) return structs[ty_sidx(t)].size;
        return ty_size(t);
    }
    // a new StructTy from its fields; returns its type
    OCB_HD Ty add_struct(Str name, const SField *f, uint32_t nf) {
        StructDef d{name, sfields.n, nf, 0};
        uint64_t total = 0;
        for (uint32_t i = 0; i < nf; ++i) {
            sfields.push(*ar, f[i]);
            uint32_t sz = tsize(f[i].ty);
            if (sz) total = (total + sz - 1) / sz * sz;
            total += sz;
        }
        d.size = total > 0x7FFFFFFFu ? 0x7FFFFFFFu : (uint32_t)total;
        if (total > 0x7FFFFFFFu) unsup = true;
        structs.push(*ar, d);
        return ty_struct(structs.n - 1);
    }
    // index of a field of struct type t, or -1 (KeyError in the reference)
    OCB_HD int32_t field_index(Ty t, Str fname) const {
        const StructDef &d = structs[ty_sidx(t)];
        for (uint32_t i = 0; i < d.nf; ++i)
            if (eq(sfields[d.f0 + i].name, fname)) return (int32_t)i;
        return -1;
    }
    OCB_HD const SField &field(Ty t, uint32_t i) const { return sfields[structs[ty_sidx(t)].f0 + i]; }
    // .align of a struct array in PTX: the largest field size (4 without
    // fields) rounded up to a power of two, at most 16 (codegen/emit.py:1013-1022)
    OCB_HD uint32_t struct_align(Ty t) const {
        const StructDef &d = structs[ty_sidx(t)];
        uint32_t mx = 0;
        for (uint32_t i = 0; i < d.nf; ++i) {
            uint32_t z = tsize(sfields[d.f0 + i].ty);
            if (i == 0 || z > mx) mx = z;
        }
        if (!d.nf) mx = 4;
        uint32_t sa = 1;
        while (sa < mx && sa < 16) sa <<= 1;
        return sa;
    }
    OCB_HD uint32_t nfields(Ty t) const { return structs[ty_sidx(t)].nf; }
    // StructTy.field_offset (types.py:126-136) of field i
    OCB_HD uint32_t field_offset(Ty t, uint32_t fi) const {
        const StructDef &d = structs[ty_sidx(t)];
        uint64_t off = 0;
        for (uint32_t i = 0; i < d.nf; ++i) {
            uint32_t sz = tsize(sfields[d.f0 + i].ty);
            if (sz) off = (off + sz - 1) / sz * sz;
            if (i == fi) break;
            off += sz;
        }
        return (uint32_t)off;
    }
    OCB_HD uint32_t add_val(uint32_t id, Ty ty, Str name) {
        if (!vals.push(*ar, Value{id, ty, name}) && vals.n == 0) return 0;
        return vals.n ? vals.n - 1 : 0;
    }
    OCB_HD Opnd cint(Ty ty, pyint v) {
        Const c{ty, 0, v, 0.0};
        consts.push(*ar, c);
        return oc(consts.n - 1);
    }
    OCB_HD Opnd cfloat(Ty ty, double v) {
        Const c{ty, 1, 0, v};
        consts.push(*ar, c);
        return oc(consts.n - 1);
    }
    // Const(ty, 0.0 if ty.is_float else 0)
    OCB_HD Opnd czero(Ty ty) { return ty_is_float(ty) ? cfloat(ty, 0.0) : cint(ty, 0); }
    OCB_HD Ty opty(Opnd o) const {
        if (o.k == O_VAL) return vals[o.x].ty;
        if (o.k == O_CONST) return consts[o.x].ty;
        if (o.k == O_SYM) return gvars[o.x].ptr;
        return S_VOID;
    }
    OCB_HD uint32_t new_block(Str label) {
        Block b;
        b.label = label;
        b.insts.init();
        b.term = Term{T_NONE, onone(), Str{nullptr, 0}, Str{nullptr, 0}};
        blocks.push(*ar, b);
        return blocks.n - 1;
    }
    OCB_HD uint32_t add_inst(const Inst &i) {
        insts.push(*ar, i);
        return insts.n - 1;
    }
};

// A set of names (the reference's per-block scope sets); order irrelevant.
struct NameSet {
    Vec<Str> v;
    OCB_HD void init() { v.init(); }
    OCB_HD void add(Arena &a, Str s) {
        for (uint32_t i = 0; i < v.n; ++i)
            if (eq(v.p[i], s)) return;
        v.push(a, s);
    }
    OCB_HD bool has(Str s) const {
        for (uint32_t i = 0; i < v.n; ++i)
            if (eq(v.p[i], s)) return true;
        return false;
    }
};

// --- intrinsic name tables of _parse_primary_expr (parser.py:1929-2033) ---
// Each list is one space-delimited string, so it lives in code on host and device.
OCB_HD inline bool in_list(Str n, const char *l) {
    for (uint32_t i = 0; l[i]; ++i) {
        if (l[i] != ' ') continue;
        uint32_t j = 0;
        while (j < n.n && l[i + 1 + j] == n.p[j]) ++j;
        if (j == n.n && n.n && l[i + 1 + j] == ' ') return true;
    }
    return false;
}
OCB_HD inline bool contains(Str s, const char *sub) {
    uint32_t k = cstrlen(sub);
    for (uint32_t i = 0; i + k <= s.n; ++i) {
        uint32_t j = 0;
        while (j < k && s.p[i + j] == sub[j]) ++j;
        if (j == k) return true;
    }
    return false;
}
#define kTexFetch " tex1Dfetch tex2D tex3D "
#define kSurfVoid " surf1Dwrite "
#define kVoidStmts " __threadfence __threadfence_block __threadfence_system __nanosleep __trap __brkpt "
#define kSyncReduce " __syncthreads_count __syncthreads_and __syncthreads_or "
#define kIntOps " __popc __popcll __clz __clzll __brev __brevll __ffs __ffsll "
#define kPredInt " isnan isinf isfinite __isnan __isinf __isfinite __isnanf __isinff __isfinitef "
#define kFloat2Int                                                                          \
    " __float2int_rn __float2int_rd __float2int_ru __float2int_rz __float2uint_rn"          \
    " __float2uint_rd __float2uint_ru __float2uint_rz __float2ll_rn __float2ll_rd"          \
    " __float2ll_ru __float2ll_rz __float2ull_rn __float2ull_rd __float2ull_ru"             \
    " __float2ull_rz __double2int_rn __double2int_rz __double2uint_rn __double2uint_rz"     \
    " __double2ll_rn __double2ll_rz __double2ull_rn __double2ull_rz __float_as_int"         \
    " __float_as_uint __double_as_longlong __double_as_ulonglong "
#define kInt2Float                                                                          \
    " __int2float_rn __int2float_rd __int2float_ru __int2float_rz __uint2float_rn"          \
    " __uint2float_rd __uint2float_ru __uint2float_rz __ll2float_rn __ll2float_rz"          \
    " __ull2float_rn __ull2float_rz __int2double_rn __ll2double_rn __uint2double_rn"        \
    " __ull2double_rn __int_as_float __uint_as_float __longlong_as_double"                  \
    " __ulonglong_as_double "
#define kWarpReduceInt " __reduce_add_sync __reduce_min_sync __reduce_max_sync "
#define kWarpReduceUint " __reduce_and_sync __reduce_or_sync __reduce_xor_sync __reduce_umin_sync __reduce_umax_sync "
#define kIntBinary2 " __mul24 __mulhi "
#define kUintBinary2 " __umul24 __umulhi __rhadd __byte_perm __funnelshift_l __funnelshift_r __funnelshift_lc __funnelshift_rc "
#define kHalfUnary                                                                          \
    " __habs __hneg __hsqrt __hrcp __hrsqrt __hexp __hlog __hceil __hfloor __hrint"         \
    " __htrunc __hcos __hsin __hexp2 __hlog2 __hlog10 __half2float __low2float"             \
    " __high2float "
#define kHalfBinary " __hmul __hmul_rn __hmul_sat __hadd_rn __hsub __hsub_rn __hdiv __hfmin __hfmax __hmin __hmax "
#define kHalfTernary " __hfma __hfma_sat __hfma_relu "
#define kHalfCmpInt " __hgt __hlt __hge __hle __heq __hne __hisnan __hisinf "
#define kHalfCvt                                                                            \
    " __float2half __float2half_rn __float2half_rd __float2half_ru __float2half_rz"         \
    " __int2half_rn __int2half_rd __int2half_ru __int2half_rz __uint2half_rn"               \
    " __uint2half_rd __uint2half_ru __uint2half_rz __short2half_rn __ushort2half_rn"        \
    " __ll2half_rn __ll2half_rz __ull2half_rn __ull2half_rz __ushort_as_half"               \
    " __short_as_half "
#define kHalf2Int                                                                           \
    " __half2int_rn __half2int_rz __half2uint_rn __half2uint_rz __half2short_rn"            \
    " __half2short_rz __half2ushort_rn __half2ushort_rz __half2ll_rn __half2ll_rz"          \
    " __half2ull_rn __half2ull_rz "
#define kFloatUnary                                                                         \
    " sqrtf rsqrtf rcpf fabsf sinf cosf tanf expf exp2f exp10f logf log2f log10f"           \
    " floorf ceilf roundf truncf atanf asinf acosf sqrt rsqrt fabs sin cos exp exp2"        \
    " exp10 log log2 log10 floor ceil round trunc atan asin acos __fsqrt_rn __fsqrt_rd"     \
    " __fsqrt_ru __fsqrt_rz __frcp_rn __frcp_rd __frcp_ru __frcp_rz __frsqrt_rn "
#define kFloatBinary " fminf fmaxf fmodf powf fmin fmax fmod pow hypotf atan2f "
#define kFloatTernary " fmaf fma __fmaf_rn __fmaf_rd __fmaf_ru __fmaf_rz __fma_rn __fma_rd __fma_ru __fma_rz "

OCB_HD inline Inst mk_inst(uint8_t kind, uint8_t op, int32_t dest, Opnd a, Opnd b) {
    Inst i;
    i.kind = kind;
    i.op = op;
    i.dest = dest;
    i.a = a;
    i.b = b;
    i.c = onone();
    i.func = Str{nullptr, 0};
    i.pidx = 0;
    i.args.init();
    return i;
}

}  // namespace cc
}  // namespace ocb
