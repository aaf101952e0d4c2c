// Parser, recursive __device__ functions: the recursion detection of
// parse_module (opencuda/frontend/parser.py:4392-4435) and
// _compile_device_func (:4089-4153), which turns each function on a call
// cycle into its own IR function (emitted as a PTX .func and called with
// call.uni) instead of expanding it at the call.
//
// The reference walks Python sets here: the callee set of each function and
// the set of functions on a cycle.  Which cycles its depth-first search finds
// and the order the functions are compiled in (their order in the PTX module)
// follow those sets' iteration order, which CPython derives from the string
// hashes (fixed by PYTHONHASHSEED=0, under which the reference runs).  So this
// file restates the string hash and the set table to get the same order.
#pragma once
#include "cc_parse_struct.cuh"

namespace ocb {
namespace cc {

// CPython's str hash with hash randomization off (PYTHONHASHSEED=0): SipHash
// with one compression and three finalization rounds (Aumasson & Bernstein's
// SipHash-c-d with c=1, d=3) under the all-zero key, over the string's bytes;
// -1 is mapped to -2.  Valid for ASCII strings (one byte per code point).
OCB_HD inline uint64_t sip_rotl(uint64_t x, int b) { return (x << b) | (x >> (64 - b)); }
OCB_HD inline int64_t py_str_hash(Str s) {
    if (s.n == 0) return 0;
    uint64_t v0 = 0x736f6d6570736575ull, v1 = 0x646f72616e646f6dull;
    uint64_t v2 = 0x6c7967656e657261ull, v3 = 0x7465646279746573ull;
    auto round = [&]() {
        v0 += v1; v1 = sip_rotl(v1, 13); v1 ^= v0; v0 = sip_rotl(v0, 32);
        v2 += v3; v3 = sip_rotl(v3, 16); v3 ^= v2;
        v0 += v3; v3 = sip_rotl(v3, 21); v3 ^= v0;
        v2 += v1; v1 = sip_rotl(v1, 17); v1 ^= v2; v2 = sip_rotl(v2, 32);
    };
    uint32_t n = s.n, i = 0;
    for (; i + 8 <= n; i += 8) {
        uint64_t mi = 0;
        for (int q = 7; q >= 0; --q) mi = (mi << 8) | (uint8_t)s.p[i + q];
        v3 ^= mi;
        round();
        v0 ^= mi;
    }
    uint64_t b = (uint64_t)n << 56;
    for (uint32_t q = 0; i + q < n; ++q) b |= (uint64_t)(uint8_t)s.p[i + q] << (8 * q);
    v3 ^= b;
    round();
    v0 ^= b;
    v2 ^= 0xff;
    round();
    round();
    round();
    int64_t h = (int64_t)((v0 ^ v1) ^ (v2 ^ v3));
    return h == -1 ? -2 : h;
}

// A CPython set of small-integer keys with given hashes (Objects/setobject.c):
// 8 slots to start; a key goes to slot hash & mask, else the next 9 slots
// when they exist, else perturbed steps i = 5i + 1 + (perturb >>= 5); the
// table grows to 4x the used count when 3/5 full.  Iteration is slot order.
struct PySet {
    Vec<int64_t> hs;
    Vec<int32_t> ks;  // -1 empty
    uint32_t mask, fill, used;

    OCB_HD bool init(Arena &a, uint32_t size = 8) {
        hs.init();
        ks.init();
        if (!hs.reserve(a, size) || !ks.reserve(a, size)) return false;
        hs.n = ks.n = size;
        for (uint32_t i = 0; i < size; ++i) {
            hs.p[i] = 0;
            ks.p[i] = -1;
        }
        mask = size - 1;
        fill = used = 0;
        return true;
    }
    OCB_HD bool has(int32_t key) const {
        for (uint32_t i = 0; i <= mask; ++i)
            if (ks.p[i] == key) return true;
        return false;
    }
    OCB_HD void insert_clean(int32_t key, int64_t hash) {
        uint64_t perturb = (uint64_t)hash;
        uint64_t i = (uint64_t)hash & mask;
        for (;;) {
            if (ks.p[i] == -1) break;
            bool put = false;
            if (i + 9 <= mask) {
                for (uint32_t j = 1; j <= 9; ++j)
                    if (ks.p[i + j] == -1) {
                        i += j;
                        put = true;
                        break;
                    }
            }
            if (put) break;
            perturb >>= 5;
            i = (i * 5 + 1 + perturb) & mask;
        }
        ks.p[i] = key;
        hs.p[i] = hash;
    }
    OCB_HD bool add(Arena &a, int32_t key, int64_t hash) {
        uint64_t perturb = (uint64_t)hash;
        uint64_t i = (uint64_t)hash & mask;
        for (;;) {
            uint32_t probes = (i + 9 <= mask) ? 9 : 0;
            uint64_t j = i;
            for (;;) {
                if (ks.p[j] == -1) {
                    ks.p[j] = key;
                    hs.p[j] = hash;
                    fill++;
                    used++;
                    if ((uint64_t)fill * 5 < (uint64_t)mask * 3) return true;
                    return resize(a, used > 50000 ? used * 2 : used * 4);
                }
                if (hs.p[j] == hash && ks.p[j] == key) return true;
                if (probes-- == 0) break;
                j++;
            }
            perturb >>= 5;
            i = (i * 5 + 1 + perturb) & mask;
        }
    }
    OCB_HD bool resize(Arena &a, uint32_t minused) {
        uint32_t ns = 8;
        while (ns <= minused) ns <<= 1;
        PySet old = *this;
        if (!init(a, ns)) return false;
        for (uint32_t q = 0; q <= old.mask; ++q)
            if (old.ks.p[q] != -1) insert_clean(old.ks.p[q], old.hs.p[q]);
        fill = used = old.used;
        return true;
    }
};

// The functions on a call cycle, in the iteration order of the reference's
// `on_cycle` set; `out` receives indices into dfuncs (each name's latest
// definition).  False when a name is outside what the hash restatement
// covers (non-ASCII).
OCB_HD inline bool Parser::recursive_funcs(Vec<uint32_t> &out) {
    out.init();
    // _device_funcs as a dict: first-definition order, latest definition
    Vec<uint32_t> uniq;  // dfuncs index of the first definition of each name
    uniq.init();
    for (uint32_t i = 0; i < dfuncs.n; ++i) {
        bool seen = false;
        for (uint32_t j = 0; j < uniq.n && !seen; ++j) seen = eq(dfuncs[uniq[j]].name, dfuncs[i].name);
        if (!seen) uniq.push(ar, i);
    }
    uint32_t n = uniq.n;
    if (!n) return true;
    Vec<int64_t> hash;
    hash.init();
    for (uint32_t j = 0; j < n; ++j) {
        Str nm = dfuncs[uniq[j]].name;
        for (uint32_t q = 0; q < nm.n; ++q)
            if ((uint8_t)nm.p[q] >= 0x80) return false;
        hash.push(ar, py_str_hash(nm));
    }
    auto name_index = [&](Str v) -> int32_t {
        for (uint32_t j = 0; j < n; ++j)
            if (eq(dfuncs[uniq[j]].name, v)) return (int32_t)j;
        return -1;
    };
    // call_graph: the set of function names among each body's identifiers
    Vec<PySet> callees;
    callees.init();
    for (uint32_t j = 0; j < n && !ar.oom; ++j) {
        PySet s;
        if (!s.init(ar)) return true;
        const DevFunc &f = dfuncs[(uint32_t)find_dfunc(dfuncs[uniq[j]].name)];
        for (uint32_t t = f.body_start; t < f.body_end && t < tk.n; ++t) {
            if (kind_at(t) != TK_IDENT) continue;
            int32_t c = name_index(val_at(t));
            if (c >= 0 && !s.add(ar, c, hash[(uint32_t)c])) return true;
        }
        callees.push(ar, s);
    }
    if (ar.oom) return true;
    // _dfs_cycle with an explicit stack; color 0 white, 1 gray, 2 black
    uint8_t *color = (uint8_t *)ar.alloc(n, 1);
    uint32_t *cursor = (uint32_t *)ar.alloc(4ull * n, 4);
    uint32_t *path = (uint32_t *)ar.alloc(4ull * n, 4);
    if (!color || !cursor || !path) return true;
    for (uint32_t j = 0; j < n; ++j) color[j] = 0;
    PySet on_cycle;
    if (!on_cycle.init(ar)) return true;
    for (uint32_t root = 0; root < n; ++root) {
        if (color[root]) continue;
        uint32_t sp = 0;
        path[sp] = root;
        cursor[sp] = 0;
        color[root] = 1;
        ++sp;
        while (sp) {
            uint32_t node = path[sp - 1];
            PySet &cs = callees[node];
            uint32_t &c = cursor[sp - 1];
            while (c <= cs.mask && cs.ks.p[c] == -1) ++c;
            if (c > cs.mask) {  // path.pop(); color = BLACK
                color[node] = 2;
                --sp;
                continue;
            }
            uint32_t nxt = (uint32_t)cs.ks.p[c++];
            if (color[nxt] == 1) {
                uint32_t idx = 0;
                while (path[idx] != nxt) ++idx;
                for (uint32_t q = idx; q < sp; ++q)
                    if (!on_cycle.add(ar, (int32_t)path[q], hash[path[q]])) return true;
            } else if (color[nxt] == 0) {
                color[nxt] = 1;
                path[sp] = nxt;
                cursor[sp] = 0;
                ++sp;
            }
        }
    }
    for (uint32_t q = 0; q <= on_cycle.mask; ++q)
        if (on_cycle.ks.p[q] != -1)
            out.push(ar, (uint32_t)find_dfunc(dfuncs[uniq[(uint32_t)on_cycle.ks.p[q]]].name));
    return true;
}

// _compile_device_func (parser.py:4089-4153): the body parsed as its own
// function (parameters as ParamInst, `return v` as a returning terminator),
// the parser's state saved around it.
OCB_HD inline void Parser::compile_devfn(uint32_t fi) {
    DevFunc f = dfuncs[fi];
    if (ty_is_struct(f.ret)) { unsup(); return; }
    for (uint32_t i = 0; i < f.params.n; ++i)
        if (ty_is_struct(f.params[i].ty)) { unsup(); return; }
    uint32_t saved_pos = pos, saved_bc = block_count, saved_cur = cur;
    VarMap saved_vars = vars;
    Kernel *saved_kern = kern;
    int32_t saved_dest = inline_dest;
    Str saved_merge = inline_merge;
    Vec<NameSet> saved_scopes = scopes;
    Kernel kk;
    kk.name = f.name;
    kk.params = f.params;
    kk.blocks.init();
    kk.next_id = 0;
    kk.n_launch = 0;
    kk.shared.init();
    kk.locals.init();
    kk.has_locals = false;
    kk.ret = f.ret;
    if (!m.funcs.push(ar, kk)) return;
    kern = &m.funcs.back();
    vars.init();
    block_count = 0;
    inline_dest = -1;
    inline_merge = Str{nullptr, 0};
    scopes.init();
    cur = new_block("entry");
    for (uint32_t i = 0; i < f.params.n && !bad(); ++i) {
        uint32_t v = new_val(f.params[i].name, f.params[i].ty);
        Inst pi = mk_inst(I_PARAM, 0, (int32_t)v, onone(), onone());
        pi.pidx = i;
        pi.func = f.params[i].name;
        emit(pi);
        vars.set(ar, f.params[i].name, ov(v));
    }
    pos = f.body_start;
    if (!expect(TK_LBRACE)) return;
    while (!bad() && !at(TK_RBRACE) && !at(TK_EOF)) parse_stmt();
    if (bad()) return;
    if (at(TK_RBRACE)) advance();
    if (B().term.kind == T_NONE) B().term = Term{T_RET, onone(), Str{nullptr, 0}, Str{nullptr, 0}};
    pos = saved_pos;
    vars = saved_vars;
    kern = saved_kern;
    block_count = saved_bc;
    cur = saved_cur;
    inline_dest = saved_dest;
    inline_merge = saved_merge;
    scopes = saved_scopes;
}

}  // namespace cc
}  // namespace ocb
