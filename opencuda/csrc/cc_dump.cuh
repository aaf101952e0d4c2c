// Canonical IR text of one TU, byte-compatible with the dump the reference's
// IR objects produce under the oracle's ir_dump (same line grammar):
//   kernel <name> next_id=<n> / launch / param / shared / local / block /
//   instruction lines / term lines.
#pragma once
#include "cc_ir.cuh"

namespace ocb {
namespace cc {

struct Out {  // bounded text sink
    char *p;
    uint64_t n, cap;
    bool full;
    OCB_HD void put(char c) {
        if (n < cap) p[n++] = c;
        else full = true;
    }
    OCB_HD void put(const char *s) {
        while (*s) put(*s++);
    }
    OCB_HD void put(Str s) {
        for (uint32_t i = 0; i < s.n; ++i) put(s.p[i]);
    }
    OCB_HD void put_i64(int64_t v) {
        char t[24];
        int k = 0;
        uint64_t u = v < 0 ? (uint64_t)0 - (uint64_t)v : (uint64_t)v;
        do {
            t[k++] = (char)('0' + u % 10);
            u /= 10;
        } while (u);
        if (v < 0) put('-');
        while (k) put(t[--k]);
    }
    OCB_HD void put_i128(pyint v) {
        char t[48];
        int k = 0;
        unsigned __int128 u = v < 0 ? (unsigned __int128)0 - (unsigned __int128)v : (unsigned __int128)v;
        do {
            t[k++] = (char)('0' + (int)(u % 10));
            u /= 10;
        } while (u);
        if (v < 0) put('-');
        while (k) put(t[--k]);
    }
    OCB_HD void put_hex64(uint64_t v) {
        const char *h = "0123456789abcdef";
        for (int s = 60; s >= 0; s -= 4) put(h[(v >> s) & 15]);
    }
};

OCB_HD inline void dump_ty(Out &o, const Module &m, Ty t) {
    if (ty_is_struct(t)) {
        o.put("struct(");
        o.put(m.structs[ty_sidx(t)].name);
        o.put(')');
        return;
    }
    if (!is_ptr(t)) {
        o.put(scalar_name(ty_scalar(t)));
        return;
    }
    o.put("ptr(");
    dump_ty(o, m, ty_pointee(t));
    o.put(',');
    o.put(as_name(ty_as(t)));
    o.put(ty_vol(t) ? ",1)" : ",0)");
}

OCB_HD inline void dump_opnd(Out &o, const Module &m, Opnd x) {
    if (x.k == O_NONE) {
        o.put('_');
        return;
    }
    if (x.k == O_VAL) {
        const Value &v = m.vals[x.x];
        o.put('%');
        o.put_i64(v.id);
        o.put(':');
        o.put(v.name);
        o.put(':');
        dump_ty(o, m, v.ty);
        return;
    }
    if (x.k == O_SYM) {
        o.put('@');
        o.put(m.gvars[x.x].name);
        return;
    }
    const Const &c = m.consts[x.x];
    o.put('#');
    dump_ty(o, m, c.ty);
    if (c.pyfloat) {
        uint64_t bits;
        memcpy(&bits, &c.f, 8);
        o.put(":f:");
        o.put_hex64(bits);
    } else {
        o.put(":i:");
        o.put_i128(c.i);
    }
}

OCB_HD inline void dump_inst(Out &o, const Module &m, const Inst &i) {
    auto dest = [&]() {
        if (i.dest < 0) o.put('_');
        else dump_opnd(o, m, ov((uint32_t)i.dest));
        o.put(" = ");
    };
    switch (i.kind) {
    case I_BIN:
    case I_CMP:
        dest();
        o.put(i.kind == I_BIN ? "bin " : "cmp ");
        o.put(i.kind == I_BIN ? binop_name(i.op) : cmpop_name(i.op));
        o.put(' ');
        dump_opnd(o, m, i.a);
        o.put(", ");
        dump_opnd(o, m, i.b);
        break;
    case I_SELECT:
        dest();
        o.put("select ");
        dump_opnd(o, m, i.c);
        o.put(", ");
        dump_opnd(o, m, i.a);
        o.put(", ");
        dump_opnd(o, m, i.b);
        break;
    case I_LOAD:
        dest();
        o.put("load ");
        dump_opnd(o, m, i.a);
        break;
    case I_STORE:
        o.put("store ");
        dump_opnd(o, m, i.a);
        o.put(", ");
        dump_opnd(o, m, i.b);
        break;
    case I_CVT:
        dest();
        o.put("cvt ");
        dump_opnd(o, m, i.a);
        break;
    case I_CALL:
        dest();
        o.put("call ");
        o.put(i.func);
        o.put('(');
        for (uint32_t k = 0; k < i.args.n; ++k) {
            if (k) o.put(", ");
            dump_opnd(o, m, i.args[k]);
        }
        o.put(')');
        break;
    case I_PRINTF:
    case I_ASM: {
        const char *h = "0123456789abcdef";
        o.put(i.kind == I_PRINTF ? "printf " : "asm ");
        for (uint32_t k = 0; k < i.func.n; ++k) {
            o.put(h[(uint8_t)i.func.p[k] >> 4]);
            o.put(h[(uint8_t)i.func.p[k] & 15]);
        }
        o.put('(');
        for (uint32_t k = 0; k < i.args.n; ++k) {
            if (i.kind == I_ASM && k == i.pidx) o.put("; ");
            else if (k) o.put(", ");
            dump_opnd(o, m, i.args[k]);
        }
        if (i.kind == I_ASM && i.pidx == i.args.n) o.put("; ");
        o.put(')');
        break;
    }
    case I_GADDR:
        dest();
        o.put("gaddr @");
        o.put(i.func);
        o.put(' ');
        o.put(as_name(i.op));
        break;
    case I_PARAM:
        dest();
        o.put("param ");
        o.put_i64(i.pidx);
        o.put(' ');
        o.put(i.func);
        break;
    }
}

OCB_HD inline void dump_term(Out &o, const Module &m, const Term &t) {
    switch (t.kind) {
    case T_NONE: o.put("term none"); break;
    case T_RET:
        o.put("term ret");
        if (t.v.k != O_NONE) {
            o.put(' ');
            dump_opnd(o, m, t.v);
        }
        break;
    case T_BR:
        o.put("term br ");
        o.put(t.t);
        break;
    case T_CBR:
        o.put("term cbr ");
        dump_opnd(o, m, t.v);
        o.put(", ");
        o.put(t.t);
        o.put(", ");
        o.put(t.f);
        break;
    }
}

OCB_HD inline void dump_module(Out &o, const Module &m) {
    for (uint32_t ki = 0; ki < m.kernels.n; ++ki) {
        const Kernel &k = m.kernels[ki];
        if (ki) o.put('\n');
        o.put("kernel ");
        o.put(k.name);
        o.put(" next_id=");
        o.put_i64(k.next_id);
        if (k.n_launch) {
            o.put("\n launch");
            for (uint32_t i = 0; i < k.n_launch; ++i) {
                o.put(' ');
                o.put_i64(k.launch[i]);
            }
        }
        for (uint32_t i = 0; i < k.params.n; ++i) {
            o.put("\n param ");
            o.put(k.params[i].name);
            o.put(' ');
            dump_ty(o, m, k.params[i].ty);
        }
        for (uint32_t i = 0; i < k.shared.n; ++i) {
            o.put("\n shared ");
            o.put(k.shared[i].name);
            o.put(' ');
            dump_ty(o, m, k.shared[i].ty);
            o.put(' ');
            o.put_i64(k.shared[i].count);
        }
        for (uint32_t i = 0; i < k.locals.n; ++i) {
            o.put("\n local ");
            o.put(k.locals[i].name);
            o.put(' ');
            dump_ty(o, m, k.locals[i].ty);
            o.put(' ');
            o.put_i64(k.locals[i].count);
            o.put(' ');
            dump_opnd(o, m, ov(k.locals[i].val));
        }
        for (uint32_t bi = 0; bi < k.blocks.n; ++bi) {
            const Block &b = m.blocks[k.blocks[bi]];
            o.put("\n block ");
            o.put(b.label);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                o.put("\n  ");
                dump_inst(o, m, m.insts[b.insts[ii]]);
            }
            o.put("\n  ");
            dump_term(o, m, b.term);
        }
    }
    if (m.gvars.n || m.funcs.n) {
        if (m.kernels.n) o.put('\n');
        o.put("module-extras");
    }
    o.put('\n');
}

}  // namespace cc
}  // namespace ocb
