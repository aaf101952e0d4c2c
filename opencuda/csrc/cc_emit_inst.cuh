// PTX emitter, instructions and terminators: emit.py:1149-3123 (_emit_inst,
// _emit_term) and emit_kernel's peepholes and declarations (:648-1126).
#pragma once
#include "cc_emit.cuh"

namespace ocb {
namespace cc {

OCB_HD inline bool sstarts(Str s, const char *p) { return starts(s, p); }

// ---- ParamInst / BinInst (emit.py:1177-1419) ---------------------------------
OCB_HD inline void Emit::emit_bin(const Inst &in) {
    const Value &dv = V((uint32_t)in.dest);
    Ty ty = dv.ty;
    const char *ptx = ptx_type(ty);
    if (cstr_in(ptx, " s8 u8 s16 u16 ")) ptx = (cstr_eq(ptx, "s8") || cstr_eq(ptx, "s16")) ? "s32" : "u32";
    Opnd L = in.a, R = in.b;
    auto czero = [&](Opnd o) { return o.k == O_CONST && pv_eq_int(pv_of(m.consts[o.x]), 0); };
    if (in.op == BO_ADD && !is_ptr(ty)) {
        bool lz = czero(L), rz = czero(R);
        if (lz && rz) {
            SB b = sb();
            if (is_half(ty)) b.s("    cvt.rn.f16.f32 ").s(reg(in.dest)).s(", 0f00000000;");
            else if (ty_is_float(ty)) b.s("    mov.").s(ptx_type(ty)).c(' ').s(reg(in.dest)).s(", 0f00000000;");
            else b.s("    mov.").s(ptx).c(' ').s(reg(in.dest)).s(", 0;");
            put(b);
            return;
        } else if (rz && is_half(ty) && L.k == O_VAL) {
            SB b = sb();
            b.s("    mov.b16 ").s(reg(in.dest)).s(", ").s(reg(L)).c(';');
            put(b);
            return;
        } else if (lz && is_half(ty) && R.k == O_VAL) {
            SB b = sb();
            b.s("    mov.b16 ").s(reg(in.dest)).s(", ").s(reg(R)).c(';');
            put(b);
            return;
        } else if ((rz && !is_half(ty)) || (lz && R.k != O_CONST && !is_half(ty))) {
            Opnd X = rz ? L : R;
            SB b = sb();
            if (ty_is_float(ty)) {
                const char *fty = ptx_type(ty);
                Str src = coerce_to_float(X, fty);
                b.s("    mov.").s(fty).c(' ').s(reg(in.dest)).s(", ").s(src).c(';');
            } else {
                Str src = X.k == O_VAL ? coerce_to_int(X, ptx) : opnd(X, ptx, true);
                b.s("    mov.").s(ptx).c(' ').s(reg(in.dest)).s(", ").s(src).c(';');
            }
            put(b);
            return;
        }
    }
    const char *opn[] = {"add", "sub", "mul.lo", "div", "rem", "and", "or", "xor", "shl", "shr"};
    const char *pop = opn[in.op];
    if (in.op == BO_MUL && ty_is_float(ty)) pop = "mul";
    if (in.op == BO_DIV && ty_is_float(ty)) pop = cstr_eq(ptx_type(ty), "f32") ? "div.approx" : "div.rn";
    if (is_half(ty)) {
        const char *hop = in.op == BO_ADD ? "add" : in.op == BO_SUB ? "sub" : in.op == BO_MUL ? "mul" :
                          in.op == BO_DIV ? "div.approx" : "add";
        auto hopnd = [&](Opnd o) -> Str {
            if (o.k == O_CONST) {
                uint32_t t = new_value("_h_tmp", S_HALF);
                uint32_t bits;
                if (!pack_f32(pv_to_float(pv_of(m.consts[o.x])), bits)) { raise_(2); return S("?"); }
                SB b = sb();
                Str tr = reg(t);
                b.s("    cvt.rn.f16.f32 ").s(tr).s(", 0f").hex(bits, 8).c(';');
                put(b);
                return reg(t);
            }
            return opnd(o, "f16");
        };
        Str ls = hopnd(L), rs = hopnd(R);
        SB b = sb();
        b.s("    ").s(hop).s(".f16 ").s(reg(in.dest)).s(", ").s(ls).s(", ").s(rs).c(';');
        put(b);
        return;
    }
    if (in.op == BO_AND || in.op == BO_OR || in.op == BO_XOR) {
        if (L.k == O_VAL && is_pred(vid(L)) && R.k == O_VAL && is_pred(vid(R))) {
            SB b = sb();
            b.s("    ").s(opn[in.op]).s(".pred ").s(reg(in.dest)).s(", ").s(reg(L)).s(", ").s(reg(R)).c(';');
            put(b);
            return;
        }
    }
    char tyb[8];
    if (in.op == BO_AND || in.op == BO_OR || in.op == BO_XOR || in.op == BO_SHL) {
        int bits = (!is_ptr(ty) && ty_size(ty) > 2) ? (int)ty_size(ty) * 8 : 32;
        tyb[0] = 'b';
        if (bits == 64) { tyb[1] = '6'; tyb[2] = '4'; } else { tyb[1] = '3'; tyb[2] = '2'; }
        tyb[3] = 0;
        ptx = tyb;
    } else if (in.op == BO_SHR) {
        int bits = (int)ty_size(ty) * 8;
        if (bits < 32) bits = 32;
        tyb[0] = (!is_ptr(ty) && ty_is_signed(ty)) ? 's' : 'b';
        tyb[1] = bits == 64 ? '6' : '3';
        tyb[2] = bits == 64 ? '4' : '2';
        tyb[3] = 0;
        ptx = tyb;
    }
    if (is_ptr(ty) && (in.op == BO_ADD || in.op == BO_SUB)) {
        Str ls = opnd(L);
        Str rs = opnd(R);
        if (R.k == O_CONST) {
            pyint iv;
            if (!pv_to_int(pv_of(m.consts[R.x]), iv)) { unsup(); return; }
            SB b = sb();
            b.i(iv);
            rs = b.str();
        } else if (R.k == O_VAL && !is_64bit(V(R.x).ty)) {
            uint32_t rid = vid(R);
            int32_t w = widen_get(rid);
            uint32_t wide;
            if (w >= 0) {
                wide = (uint32_t)w;
            } else {
                wide = new_value(nm("wide", dv.id), ty);
                Ty rt = V(R.x).ty;
                const char *wop = (!is_ptr(rt) && ty_is_signed(rt)) ? "cvt.s64.s32" : "cvt.u64.u32";
                SB b = sb();
                b.s("    ").s(wop).c(' ').s(reg(wide)).s(", ").s(rs).c(';');
                put(b);
                widen_set(rid, wide);
            }
            rs = reg(wide);
        }
        SB b = sb();
        b.s("    ").s(pop).s(".u64 ").s(reg(in.dest)).s(", ").s(ls).s(", ").s(rs).c(';');
        put(b);
    } else if (ty_is_float(ty)) {
        const char *fty = ptx_type(ty);
        Str ls = coerce_to_float(L, fty);
        Str rs = coerce_to_float(R, fty);
        SB b = sb();
        b.s("    ").s(pop).c('.').s(fty).c(' ').s(reg(in.dest)).s(", ").s(ls).s(", ").s(rs).c(';');
        put(b);
    } else if (is_64bit(ty)) {
        auto b64 = [&](Opnd o, const char *tgt) -> Str {
            if (o.k == O_VAL && !is_64bit(V(o.x).ty)) {
                int32_t w = widen_get(vid(o));
                uint32_t wid;
                if (w < 0) {
                    Ty ot = V(o.x).ty;
                    const char *wop = (!is_ptr(ot) && ty_is_signed(ot)) ? "cvt.s64.s32" : "cvt.u64.u32";
                    wid = new_value(nm("_wide", dv.id), ty);
                    SB b = sb();
                    Str wr = reg(wid);
                    b.s("    ").s(wop).c(' ').s(wr).s(", ").s(reg(o)).c(';');
                    put(b);
                    widen_set(vid(o), wid);
                } else {
                    wid = (uint32_t)w;
                }
                return reg(wid);
            }
            return opnd(o, tgt, true);
        };
        if (in.op == BO_SHL || in.op == BO_SHR) {
            Str ls = b64(L, ptx);
            Str rs;
            if (R.k == O_VAL && is_64bit(V(R.x).ty)) {
                uint32_t nw = new_value(nm("_sham", dv.id), S_UINT32);
                SB b = sb();
                Str nr = reg(nw);
                b.s("    cvt.u32.u64 ").s(nr).s(", ").s(reg(R)).c(';');
                put(b);
                rs = reg(nw);
            } else {
                rs = opnd(R, "b32", true);
            }
            SB b = sb();
            b.s("    ").s(pop).c('.').s(ptx).c(' ').s(reg(in.dest)).s(", ").s(ls).s(", ").s(rs).c(';');
            put(b);
        } else {
            Str dr = reg(in.dest);
            Str ls = b64(L, ptx);
            Str rs = b64(R, ptx);
            SB b = sb();
            b.s("    ").s(pop).c('.').s(ptx).c(' ').s(dr).s(", ").s(ls).s(", ").s(rs).c(';');
            put(b);
        }
    } else {
        Str dr = reg(in.dest);
        Str ls = opnd(L, ptx, true);
        Str rs = opnd(R, ptx, true);
        SB b = sb();
        b.s("    ").s(pop).c('.').s(ptx).c(' ').s(dr).s(", ").s(ls).s(", ").s(rs).c(';');
        put(b);
    }
}

// ---- CmpInst (emit.py:1421-1526) -----------------------------------------------
OCB_HD inline void Emit::emit_cmp(const Inst &in) {
    Opnd L = in.a, R = in.b;
    auto czero = [&](Opnd o) { return o.k == O_CONST && pv_eq_int(pv_of(m.consts[o.x]), 0); };
    if (in.op == CO_EQ && L.k == O_VAL && is_pred(vid(L)) && czero(R)) {
        SB b = sb();
        Str p = reg(in.dest);
        b.s("    not.pred ").s(p).s(", ").s(reg(L)).c(';');
        put(b);
        return;
    }
    if (in.op == CO_EQ && R.k == O_VAL && is_pred(vid(R)) && czero(L)) {
        SB b = sb();
        Str p = reg(in.dest);
        b.s("    not.pred ").s(p).s(", ").s(reg(R)).c(';');
        put(b);
        return;
    }
    bool lp = L.k == O_VAL && is_pred(vid(L)), rp = R.k == O_VAL && is_pred(vid(R));
    if (lp && rp) {
        Str p = reg(in.dest), lr = reg(L), rr = reg(R);
        if (in.op == CO_NE) {
            SB b = sb();
            b.s("    xor.pred ").s(p).s(", ").s(lr).s(", ").s(rr).c(';');
            put(b);
        } else if (in.op == CO_EQ) {
            Str t = fresh_pred();
            SB b = sb();
            b.s("    xor.pred ").s(t).s(", ").s(lr).s(", ").s(rr).c(';');
            put(b);
            SB b2 = sb();
            b2.s("    not.pred ").s(p).s(", ").s(t).c(';');
            put(b2);
        } else {
            pred_to_int(L, "s32");
            pred_to_int(R, "s32");
            raise_(6);  // the reference raises UnboundLocalError here
        }
        return;
    }
    Ty lt = (L.k == O_VAL || L.k == O_CONST) ? m.opty(L) : (Ty)S_INT32;
    Ty rt = (R.k == O_VAL || R.k == O_CONST) ? m.opty(R) : (Ty)S_INT32;
    bool lf = ty_is_float(lt), rf = ty_is_float(rt);
    Ty ty;
    if (lf || rf) {
        if (lf && rf) ty = ty_size(lt) >= ty_size(rt) ? lt : rt;
        else ty = lf ? lt : rt;
    } else if (!is_ptr(lt) && ty_size(lt) == 8) {
        ty = lt;
    } else if (!is_ptr(rt) && ty_size(rt) == 8) {
        ty = rt;
    } else if (!is_ptr(lt) && !is_ptr(rt) && !ty_is_signed(lt)) {
        ty = lt;
    } else if (!is_ptr(lt) && !is_ptr(rt) && !ty_is_signed(rt)) {
        ty = rt;
    } else {
        ty = lt;
    }
    const char *ptx = ptx_type(ty);
    if (cstr_in(ptx, " s8 u8 s16 u16 ")) ptx = (cstr_eq(ptx, "s8") || cstr_eq(ptx, "s16")) ? "s32" : "u32";
    bool isf = ty_is_float(ty);
    const char *cn[] = {"eq", isf ? "neu" : "ne", "lt", "le", "gt", "ge"};
    const char *cmp = cn[in.op];
    Str p = reg(in.dest);
    auto co = [&](Opnd o) -> Str {
        if (o.k == O_VAL && (cstr_eq(ptx, "u64") || cstr_eq(ptx, "s64")) && !is_64bit(V(o.x).ty)) {
            int32_t w = widen_get(vid(o));
            uint32_t wid;
            if (w < 0) {
                Ty ot = V(o.x).ty;
                bool sg = !is_ptr(ot) && ty_is_signed(ot);
                wid = new_value("_cmp_wide", sg ? S_INT64 : S_UINT64);
                SB b = sb();
                Str wr = reg(wid);
                b.s("    ").s(sg ? "cvt.s64.s32" : "cvt.u64.u32").c(' ').s(wr).s(", ").s(reg(o)).c(';');
                put(b);
                widen_set(vid(o), wid);
            } else {
                wid = (uint32_t)w;
            }
            return reg(wid);
        }
        return opnd(o, ptx);
    };
    Str ls = co(L);
    Str rs = co(R);
    SB b = sb();
    b.s("    setp.").s(cmp).c('.').s(ptx).c(' ').s(p).s(", ").s(ls).s(", ").s(rs).c(';');
    put(b);
}

// ---- CvtInst (emit.py:1528-1557) --------------------------------------------------
OCB_HD inline void Emit::emit_cvt(const Inst &in) {
    Opnd S_ = in.a;
    Ty st = (S_.k == O_VAL || S_.k == O_CONST) ? m.opty(S_) : (Ty)S_INT32;
    Ty dt = V((uint32_t)in.dest).ty;
    const char *dptx = ptx_type(dt);
    bool sbool = !is_ptr(st) && ty_scalar(st) == S_BOOL;
    bool spred = S_.k == O_VAL && is_pred(vid(S_));
    if (sbool || spred) {
        Str ps = opnd(S_);
        const char *t = "1", *f = "0";
        if (cstr_eq(dptx, "f32")) { t = "0f3F800000"; f = "0f00000000"; }
        else if (cstr_eq(dptx, "f64")) { t = "0d3FF0000000000000"; f = "0d0000000000000000"; }
        else if (cstr_eq(dptx, "f16")) { t = "0h3C00"; f = "0h0000"; }
        SB b = sb();
        b.s("    selp.").s(dptx).c(' ').s(reg(in.dest)).s(", ").s(t).s(", ").s(f).s(", ").s(ps).c(';');
        put(b);
        return;
    }
    const char *sptx = ptx_type(st);
    uint32_t sw = is_ptr(st) ? 8 : ty_size(st), dw = is_ptr(dt) ? 8 : ty_size(dt);
    if (sw == dw && sw <= 4 && !is_ptr(st) && !ty_is_float(st) && !ty_is_float(dt)) {
        Str so = opnd(S_, sptx, true);
        SB b = sb();
        b.s("    mov.b32 ").s(reg(in.dest)).s(", ").s(so).c(';');
        put(b);
    } else {
        const char *rnd = cvt_modifier(dt, st);
        Str so = opnd(S_, sptx, true);
        SB b = sb();
        b.s("    cvt").s(rnd).c('.').s(dptx).c('.').s(sptx).c(' ').s(reg(in.dest)).s(", ").s(so).c(';');
        put(b);
    }
}

// ---- LoadInst / StoreInst (emit.py:1593-1657) -----------------------------------
OCB_HD inline void Emit::emit_load(const Inst &in) {
    Ty ty = V((uint32_t)in.dest).ty;
    const char *ptx = ptx_type(ty);
    const char *sp = "global";
    bool nc = false, vol = false;
    if (in.a.k == O_VAL && is_ptr(V(in.a.x).ty)) {
        Ty pt = V(in.a.x).ty;
        vol = ty_vol(pt);
        uint32_t as = ty_as(pt);
        if (as == AS_SHARED) sp = "shared";
        else if (as == AS_LOCAL) sp = "local";
        else if (as == AS_CONST) nc = true;
    } else if (in.a.k == O_SYM) {  // [symbol] in the symbol's own state space
        Ty pt = m.gvars[in.a.x].ptr;
        if (ty_vol(pt)) vol = true;
        uint32_t as = ty_as(pt);
        if (as == AS_CONST) sp = "const";
        else if (as == AS_SHARED) sp = "shared";
    }
    if (cstr_eq(ptx, "f16")) ptx = "b16";
    SB b = sb();
    Str dr = reg(in.dest);
    Str ar_ = opnd(in.a);
    if (vol && (cstr_eq(sp, "global") || cstr_eq(sp, "shared")))
        b.s("    ld.volatile.").s(sp).c('.').s(ptx).c(' ').s(dr).s(", [").s(ar_).s("];");
    else if (nc)
        b.s("    ld.global.nc.").s(ptx).c(' ').s(dr).s(", [").s(ar_).s("];");
    else
        b.s("    ld.").s(sp).c('.').s(ptx).c(' ').s(dr).s(", [").s(ar_).s("];");
    put(b);
}

OCB_HD inline void Emit::emit_store(const Inst &in) {
    Ty ty = (in.b.k == O_VAL || in.b.k == O_CONST) ? m.opty(in.b) : (Ty)S_INT32;
    const char *ptx = ptx_type(ty);
    if (cstr_eq(ptx, "f16")) ptx = "b16";
    const char *sp = "global";
    bool vol = false;
    if (in.a.k == O_VAL && is_ptr(V(in.a.x).ty)) {
        Ty pt = V(in.a.x).ty;
        vol = ty_vol(pt);
        uint32_t as = ty_as(pt);
        if (as == AS_SHARED) sp = "shared";
        else if (as == AS_LOCAL) sp = "local";
    }
    Str vs = (in.b.k == O_VAL && is_pred(vid(in.b))) ? pred_to_int(in.b, ptx) : opnd(in.b, ptx);
    SB b = sb();
    Str ar_ = opnd(in.a);
    if (vol && (cstr_eq(sp, "global") || cstr_eq(sp, "shared")))
        b.s("    st.volatile.").s(sp).c('.').s(ptx).s(" [").s(ar_).s("], ").s(vs).c(';');
    else
        b.s("    st.").s(sp).c('.').s(ptx).s(" [").s(ar_).s("], ").s(vs).c(';');
    put(b);
}

// ---- CallInst (emit.py:1741-2885) -----------------------------------------------
OCB_HD inline void Emit::emit_call(const Inst &in) {
    Str f = in.func;
    uint32_t na = in.args.n;
    auto arg = [&](uint32_t i) { return in.args[i]; };
    if (sstarts(f, "__devfn_")) {  // call.uni of a recursive device function (emit.py:1744-1776)
        uint32_t n = pf_count++;
        put("    {");
        auto aty = [&](uint32_t i) -> const char * {
            Opnd a = arg(i);
            const char *t = (a.k == O_VAL || a.k == O_CONST) ? ptx_type(m.opty(a)) : "s32";
            return cstr_eq(t, "f16") ? "b16" : t;
        };
        for (uint32_t i = 0; i < na; ++i) {
            SB b = sb();
            b.s("        .param .").s(aty(i)).s(" _ca").i(i).c('_').i(n).c(';');
            put(b);
        }
        const char *rt = nullptr;
        if (in.dest >= 0) {
            rt = ptx_type(V((uint32_t)in.dest).ty);
            if (cstr_eq(rt, "f16")) rt = "b16";
            SB b = sb();
            b.s("        .param .").s(rt).s(" _cr_").i(n).c(';');
            put(b);
        }
        for (uint32_t i = 0; i < na; ++i) {
            Str src = opnd(arg(i));
            SB b = sb();
            b.s("        st.param.").s(aty(i)).s(" [_ca").i(i).c('_').i(n).s("], ").s(src).c(';');
            put(b);
        }
        SB al = sb();
        for (uint32_t i = 0; i < na; ++i) {
            if (i) al.s(", ");
            al.s("_ca").i(i).c('_').i(n);
        }
        Str args = al.str();
        if (rt) {
            SB b = sb();
            b.s("        call.uni (_cr_").i(n).s("), ").s(f).s(", (").s(args).s(");");
            put(b);
            Str d = reg(in.dest);
            SB b2 = sb();
            b2.s("        ld.param.").s(rt).c(' ').s(d).s(", [_cr_").i(n).s("];");
            put(b2);
        } else {
            SB b = sb();
            b.s("        call.uni ").s(f).s(", (").s(args).s(");");
            put(b);
        }
        put("    }");
        return;
    }
    if (eq(f, "tex1Dfetch") || eq(f, "tex2D") || eq(f, "tex3D")) {
        // texture fetch: a v4 read, the first component into dest (emit.py:1919-1952)
        Str dest = in.dest >= 0 ? reg(in.dest) : S("%f0");
        Str tex = na ? opnd(arg(0)) : S("%rd0");
        int dim = eq(f, "tex1Dfetch") ? 1 : eq(f, "tex2D") ? 2 : 3;
        Str c[3];
        if (dim == 1) {
            c[0] = na > 1 ? opnd(arg(1)) : S("0");
        } else {
            for (int q = 0; q < dim; ++q) c[q] = na > (uint32_t)q + 1 ? opnd(arg(q + 1)) : S("0f00000000");
        }
        uint32_t n = in.dest >= 0 ? V((uint32_t)in.dest).id : 0;
        uint32_t f1 = new_value(nm("_tex_g_", n), S_FLOAT), f2 = new_value(nm("_tex_b_", n), S_FLOAT),
                 f3 = new_value(nm("_tex_a_", n), S_FLOAT);
        Str r1 = reg(f1), r2 = reg(f2), r3 = reg(f3);
        SB b = sb();
        b.s(dim == 1 ? "    tex.1d.v4.f32.s32 {" : dim == 2 ? "    tex.2d.v4.f32.f32 {" : "    tex.3d.v4.f32.f32 {")
            .s(dest).s(", ").s(r1).s(", ").s(r2).s(", ").s(r3).s("}, [").s(tex).s(", {").s(c[0]);
        if (dim == 2) b.s(", ").s(c[1]);
        if (dim == 3) b.s(", ").s(c[1]).s(", ").s(c[2]).s(", ").s(c[2]);
        b.s("}];");
        put(b);
        return;
    }
    if (eq(f, "surf1Dread")) {  // (emit.py:1953-1958)
        Str dest = in.dest >= 0 ? reg(in.dest) : S("%r0");
        Str surf = na ? opnd(arg(0)) : S("%rd0");
        Str c = na > 1 ? opnd(arg(1)) : S("0");
        SB b = sb();
        b.s("    suld.b.1d.b32.trap {").s(dest).s("}, [").s(surf).s(", {").s(c).s("}];");
        put(b);
        return;
    }
    if (eq(f, "surf1Dwrite")) {  // (emit.py:1959-1964)
        Str v = na ? opnd(arg(0)) : S("0");
        Str surf = na > 1 ? opnd(arg(1)) : S("%rd0");
        Str c = na > 2 ? opnd(arg(2)) : S("0");
        SB b = sb();
        b.s("    sust.b.1d.b32.trap [").s(surf).s(", {").s(c).s("}], {").s(v).s("};");
        put(b);
        return;
    }
    if (eq(f, "__mbarrier_init")) {  // (emit.py:1985-1989)
        Str mb = na ? opnd(arg(0)) : S("%rd0");
        Str cnt = na > 1 ? opnd(arg(1)) : S("1");
        SB b = sb();
        b.s("    mbarrier.init.shared::cta.b64 [").s(mb).s("], ").s(cnt).c(';');
        put(b);
        return;
    }
    if (eq(f, "__mbarrier_try_wait_parity")) {  // (emit.py:1990-1999)
        Str dest = in.dest >= 0 ? reg(in.dest) : S("%r0");
        Str mb = na ? opnd(arg(0)) : S("%rd0");
        Str ph = na > 1 ? opnd(arg(1)) : S("0");
        uint32_t n = in.dest >= 0 ? V((uint32_t)in.dest).id : 0;
        uint32_t pt = new_value(nm("_mbar_p_", n), S_BOOL);
        add_pred(V(pt).id);
        Str pr = reg(pt);
        SB b = sb();
        b.s("    mbarrier.try_wait.parity.shared::cta.b64 ").s(pr).s(", [").s(mb).s("], ").s(ph).c(';');
        put(b);
        SB b2 = sb();
        b2.s("    selp.s32 ").s(dest).s(", 1, 0, ").s(pr).c(';');
        put(b2);
        return;
    }
    if (sstarts(f, "atomic")) {
        const char *aop = eq(f, "atomicAdd") ? "add" : eq(f, "atomicMin") ? "min" :
                          eq(f, "atomicMax") ? "max" : eq(f, "atomicAnd") ? "and" :
                          eq(f, "atomicOr") ? "or" : eq(f, "atomicXor") ? "xor" :
                          eq(f, "atomicExch") ? "exch" : eq(f, "atomicCAS") ? "cas" :
                          eq(f, "atomicInc") ? "inc" : eq(f, "atomicDec") ? "dec" : "add";
        Str addr = na ? opnd(arg(0)) : S("%rd0");
        const char *sp = "global";
        if (na && arg(0).k == O_VAL && is_ptr(V(arg(0).x).ty) && ty_as(V(arg(0).x).ty) == AS_SHARED) sp = "shared";
        const char *vt = "u32";
        if (na > 1 && (arg(1).k == O_VAL || arg(1).k == O_CONST)) vt = ptx_type(m.opty(arg(1)));
        if (eq(f, "atomicAdd") && cstr_eq(vt, "s64")) vt = "u64";
        if (eq(f, "atomicAnd") || eq(f, "atomicOr") || eq(f, "atomicXor") || eq(f, "atomicExch")) {
            if (cstr_eq(vt, "s32") || cstr_eq(vt, "u32")) vt = "b32";
            else if (cstr_eq(vt, "s64") || cstr_eq(vt, "u64")) vt = "b64";
        }
        Str dest = in.dest >= 0 ? reg(in.dest) : S("%r0");
        bool vtf = false;
        for (const char *q = vt; *q; ++q) vtf |= *q == 'f';
        if (eq(f, "atomicSub")) {
            if (na < 2) { unsup(); return; }
            Opnd va = arg(1);
            if (va.k == O_CONST) {
                PyVal v = pv_of(m.consts[va.x]);
                SB nb = sb();
                if (!vtf) {
                    PyVal neg = v.isf ? pv_float(-v.f) : pv_int(-v.i);
                    pyint iv;
                    if (!pv_to_int(neg, iv)) { unsup(); return; }
                    nb.i(iv);
                } else {
                    uint32_t bits;
                    if (!pack_f32(-pv_to_float(v), bits)) { raise_(2); return; }
                    nb.s("0f").hex(bits, 8);
                }
                SB b = sb();
                b.s("    atom.").s(sp).s(".add.").s(vt).c(' ').s(dest).s(", [").s(addr).s("], ").s(nb.str()).c(';');
                put(b);
            } else {
                SB n = sb();
                n.s("_neg_");
                if (in.dest >= 0) n.i(V((uint32_t)in.dest).id);
                else n.c('x');
                uint32_t nt = new_value(n.str(), m.opty(va));
                SB b = sb();
                Str nr = reg(nt);
                b.s("    sub.").s(vt).c(' ').s(nr).s(", ").s(vtf ? "0.0" : "0").s(", ").s(opnd(va, vt)).c(';');
                put(b);
                SB b2 = sb();
                b2.s("    atom.").s(sp).s(".add.").s(vt).c(' ').s(dest).s(", [").s(addr).s("], ").s(reg(nt)).c(';');
                put(b2);
            }
        } else if (eq(f, "atomicCAS")) {
            if (na < 3) { unsup(); return; }
            Opnd ca = arg(1), nw = arg(2);
            const char *ct = "b32";
            const char *cp = ptx_type(m.opty(ca));
            if (cstr_eq(cp, "s64") || cstr_eq(cp, "u64")) ct = "b64";
            SB b = sb();
            Str cs = opnd(ca, ct), ns = opnd(nw, ct);
            b.s("    atom.").s(sp).s(".cas.").s(ct).c(' ').s(dest).s(", [").s(addr).s("], ").s(cs).s(", ").s(ns).c(';');
            put(b);
        } else {
            if (na < 2) { unsup(); return; }
            SB b = sb();
            Str vs = opnd(arg(1), vt);
            b.s("    atom.").s(sp).c('.').s(aop).c('.').s(vt).c(' ').s(dest).s(", [").s(addr).s("], ").s(vs).c(';');
            put(b);
        }
        return;
    }
    if (eq(f, "__shfl_sync") || eq(f, "__shfl_up_sync") || eq(f, "__shfl_down_sync") ||
        eq(f, "__shfl_xor_sync")) {
        const char *mode = eq(f, "__shfl_sync") ? "idx" : eq(f, "__shfl_up_sync") ? "up" :
                           eq(f, "__shfl_down_sync") ? "down" : "bfly";
        Str mask = na ? opnd(arg(0)) : S("0xFFFFFFFF");
        Str val = na > 1 ? opnd(arg(1)) : S("%r0");
        Str delta = na > 2 ? opnd(arg(2)) : S("0");
        Str dest = in.dest >= 0 ? reg(in.dest) : S("%r0");
        const char *clamp = cstr_eq(mode, "up") ? "0" : "31";
        bool is64 = na > 1 && arg(1).k == O_VAL && !is_ptr(V(arg(1).x).ty) && ty_size(V(arg(1).x).ty) == 8;
        if (is64 && sstarts(dest, "%rd")) {
            uint32_t n = in.dest >= 0 ? V((uint32_t)in.dest).id : 0;
            uint32_t li = new_value(nm("_shfl_lo_in_", n), S_INT32);
            uint32_t hi = new_value(nm("_shfl_hi_in_", n), S_INT32);
            uint32_t lo = new_value(nm("_shfl_lo_out_", n), S_INT32);
            uint32_t ho = new_value(nm("_shfl_hi_out_", n), S_INT32);
            SB b = sb();
            b.s("    mov.b64 {").s(reg(li)).s(", ").s(reg(hi)).s("}, ").s(val).c(';');
            put(b);
            SB b2 = sb();
            b2.s("    shfl.sync.").s(mode).s(".b32 ").s(reg(lo)).s(", ").s(reg(li)).s(", ").s(delta).s(", ").s(clamp).s(", ").s(mask).c(';');
            put(b2);
            SB b3 = sb();
            b3.s("    shfl.sync.").s(mode).s(".b32 ").s(reg(ho)).s(", ").s(reg(hi)).s(", ").s(delta).s(", ").s(clamp).s(", ").s(mask).c(';');
            put(b3);
            SB b4 = sb();
            b4.s("    mov.b64 ").s(dest).s(", {").s(reg(lo)).s(", ").s(reg(ho)).s("};");
            put(b4);
        } else {
            SB b = sb();
            b.s("    shfl.sync.").s(mode).s(".b32 ").s(dest).s(", ").s(val).s(", ").s(delta).s(", ").s(clamp).s(", ").s(mask).c(';');
            put(b);
        }
        return;
    }
    if (eq(f, "__ballot_sync") || eq(f, "__all_sync") || eq(f, "__any_sync")) {
        Str mask = na ? opnd(arg(0)) : S("0xFFFFFFFF");
        bool have = na > 1;
        Str dest = in.dest >= 0 ? reg(in.dest) : S("%r0");
        Str tp;
        if (have && arg(1).k == O_VAL && is_pred(vid(arg(1)))) {
            tp = opnd(arg(1));
        } else {
            Str cv_ = have ? opnd(arg(1)) : S("0");
            tp = alloc_pred();
            SB b = sb();
            b.s("    setp.ne.s32 ").s(tp).s(", ").s(cv_).s(", 0;");
            put(b);
        }
        if (eq(f, "__ballot_sync")) {
            SB b = sb();
            b.s("    vote.sync.ballot.b32 ").s(dest).s(", ").s(tp).s(", ").s(mask).c(';');
            put(b);
        } else {
            Str t2 = alloc_pred();
            SB b = sb();
            b.s("    vote.sync.").s(eq(f, "__all_sync") ? "all" : "any").s(".pred ").s(t2).s(", ").s(tp).s(", ").s(mask).c(';');
            put(b);
            SB b2 = sb();
            b2.s("    selp.s32 ").s(dest).s(", 1, 0, ").s(t2).c(';');
            put(b2);
        }
        return;
    }
    if (in_list(f, " tex1Dfetch tex2D tex3D surf1Dread surf1Dwrite __cp_async_bulk_tensor_1d"
                   " __cp_async_bulk_tensor_2d __cp_async_bulk_commit_group"
                   " __cp_async_bulk_wait_group __mbarrier_init __mbarrier_try_wait_parity ")) {
        unsup();
        return;
    }
    if (eq(f, "__syncthreads")) {
        put("    bar.sync 0;");
        return;
    }
    const char *sr = nullptr;
    if (eq(f, "threadIdx.x")) sr = "tid.x";
    else if (eq(f, "threadIdx.y")) sr = "tid.y";
    else if (eq(f, "threadIdx.z")) sr = "tid.z";
    else if (eq(f, "blockIdx.x")) sr = "ctaid.x";
    else if (eq(f, "blockIdx.y")) sr = "ctaid.y";
    else if (eq(f, "blockIdx.z")) sr = "ctaid.z";
    else if (eq(f, "blockDim.x")) sr = "ntid.x";
    else if (eq(f, "blockDim.y")) sr = "ntid.y";
    else if (eq(f, "blockDim.z")) sr = "ntid.z";
    else if (eq(f, "gridDim.x")) sr = "nctaid.x";
    else if (eq(f, "gridDim.y")) sr = "nctaid.y";
    else if (eq(f, "gridDim.z")) sr = "nctaid.z";
    if (sr) {
        if (in.dest < 0) { unsup(); return; }
        SB b = sb();
        b.s("    mov.u32 ").s(reg(in.dest)).s(", %").s(sr).c(';');
        put(b);
        return;
    }
    if (sstarts(f, "threadIdx.") || sstarts(f, "blockIdx.") || sstarts(f, "blockDim.") ||
        sstarts(f, "gridDim.")) {
        // threadIdx.w etc. reach the generic branch in the reference
    }
    Str dest = in.dest >= 0 ? reg(in.dest) : S("%r0");
    emit_math(in, dest);
}

// Every call name the reference's emitter has a case for (the string
// comparisons and table lookups on CallInst.func in codegen/emit.py:1743-2885).
// A call outside this set, and not an atomic or __devfn_ name, gets no code
// there: only its destination register is taken.
__device__ __host__ inline const char *ref_call_names() {
    return
    " __activemask __all_sync __any_sync __ballot_sync __brev __brevll __brkpt __byte_perm "
    " __clock64 __clz __clzll __cp_async_bulk_commit_group __cp_async_bulk_tensor_1d "
    " __cp_async_bulk_tensor_2d __cp_async_bulk_wait_group __double2int_rn __double2int_rz "
    " __double2ll_rn __double2ll_rz __double2uint_rn __double2uint_rz __double2ull_rn "
    " __double2ull_rz __double_as_longlong __double_as_ulonglong __dp4a __dp4a_su __dp4a_u "
    " __dp4a_us __ffs __ffsll __float2half __float2half_rd __float2half_rn __float2half_ru "
    " __float2half_rz __float2int_rd __float2int_rn __float2int_ru __float2int_rz "
    " __float2ll_rd __float2ll_rn __float2ll_ru __float2ll_rz __float2uint_rd __float2uint_rn "
    " __float2uint_ru __float2uint_rz __float2ull_rd __float2ull_rn __float2ull_ru "
    " __float2ull_rz __float_as_int __float_as_uint __fma_rd __fma_rn __fma_ru __fma_rz "
    " __fmaf_rd __fmaf_rn __fmaf_ru __fmaf_rz __frcp_rd __frcp_rn __frcp_ru __frcp_rz "
    " __frsqrt_rn __fsqrt_rd __fsqrt_rn __fsqrt_ru __fsqrt_rz __funnelshift_l __funnelshift_lc "
    " __funnelshift_r __funnelshift_rc __habs __hadd __hadd_rn __hadd_sat __half2float "
    " __half2int_rn __half2int_rz __half2ll_rn __half2ll_rz __half2short_rn __half2short_rz "
    " __half2uint_rn __half2uint_rz __half2ull_rn __half2ull_rz __half2ushort_rn "
    " __half2ushort_rz __half_as_short __half_as_ushort __hceil __hcos __hdiv __heq __hexp "
    " __hexp2 __hfloor __hfma __hfma_relu __hfma_sat __hfmax __hfmin __hge __hgt __high2float "
    " __hisinf __hisnan __hle __hlog __hlog10 __hlog2 __hlt __hmax __hmin __hmul __hmul_rn "
    " __hmul_sat __hne __hneg __hrcp __hrint __hrsqrt __hsin __hsqrt __hsub __hsub_rn __htrunc "
    " __int2double_rn __int2float_rd __int2float_rn __int2float_ru __int2float_rz "
    " __int2half_rn __int2half_rz __int_as_float __isfinite __isfinitef __isinf __isinff "
    " __isnan __isnanf __ll2double_rn __ll2float_rn __ll2float_rz __ll2half_rn __ll2half_rz "
    " __longlong_as_double __low2float __match_all_sync __match_any_sync __mbarrier_init "
    " __mbarrier_try_wait_parity __mul24 __mulhi __nanosleep __popc __popcll __reduce_add_sync "
    " __reduce_and_sync __reduce_max_sync __reduce_min_sync __reduce_or_sync "
    " __reduce_umax_sync __reduce_umin_sync __reduce_xor_sync __rhadd __sad __shfl_down_sync "
    " __shfl_sync __shfl_up_sync __shfl_xor_sync __short2half_rn __short_as_half __syncthreads "
    " __syncthreads_and __syncthreads_count __syncthreads_or __syncwarp __threadfence "
    " __threadfence_block __threadfence_system __trap __uint2double_rn __uint2float_rd "
    " __uint2float_rn __uint2float_ru __uint2float_rz __uint2half_rn __uint2half_rz "
    " __uint_as_float __ull2double_rn __ull2float_rn __ull2float_rz __ull2half_rn "
    " __ull2half_rz __ulonglong_as_double __umul24 __umulhi __usad __ushort2half_rn "
    " __ushort_as_half abs acos acosf asin asinf atan atan2 atan2f atanf atomicAdd atomicAnd "
    " atomicCAS atomicExch atomicOr atomicSub atomicXor blockDim.x blockDim.y blockDim.z "
    " blockIdx.x blockIdx.y blockIdx.z cbrt cbrtf ceil ceilf clock clock64 cos cosf exp exp10 "
    " exp10f exp2 exp2f expf fabs fabsf floor floorf fma fmaf fmax fmaxf fmin fminf fmod fmodf "
    " gridDim.x gridDim.y gridDim.z hypot hypotf isfinite isinf isnan ll log log10 log10f log2 "
    " log2f logf max min pow powf rcpf round roundf rsqrt rsqrtf sin sinf sqrt sqrtf "
    " surf1Dread surf1Dwrite tan tanf tex1Dfetch tex2D tex3D threadIdx.x threadIdx.y "
    " threadIdx.z trunc truncf uint ull warpSize ";
}

// Math intrinsics and other calls (emit.py:2029-2885), the common subset.
OCB_HD inline void Emit::emit_math(const Inst &in, Str dest) {
    Str f = in.func;
    uint32_t na = in.args.n;
    auto arg = [&](uint32_t i) { return in.args[i]; };
    bool a0f64 = na && arg(0).k == O_VAL && !is_ptr(V(arg(0).x).ty) && ty_scalar(V(arg(0).x).ty) == S_DOUBLE;
    uint32_t dn = in.dest >= 0 ? V((uint32_t)in.dest).id : 0;
    auto line1 = [&](const char *op, Str d, Str a) {
        SB b = sb();
        b.s("    ").s(op).c(' ').s(d).s(", ").s(a).c(';');
        put(b);
    };
    auto arg0 = [&](const char *dflt) { return na ? opnd(arg(0)) : S(dflt); };
    if (eq(f, "__nanosleep")) {
        Str ns = na ? opnd(arg(0)) : S("0");
        SB b = sb();
        b.s("    nanosleep.u32 ").s(ns).c(';');
        put(b);
    } else if (eq(f, "__trap")) {
        put("    trap;");
    } else if (eq(f, "__brkpt")) {
        put("    brkpt;");
    } else if (eq(f, "clock64") || eq(f, "__clock64")) {
        SB b = sb();
        b.s("    mov.u64 ").s(dest).s(", %clock64;");
        put(b);
    } else if (eq(f, "clock")) {
        SB b = sb();
        b.s("    mov.u32 ").s(dest).s(", %clock;");
        put(b);
    } else if (eq(f, "__threadfence")) {
        put("    membar.gl;");
    } else if (eq(f, "__threadfence_block")) {
        put("    membar.cta;");
    } else if (eq(f, "__threadfence_system")) {
        put("    membar.sys;");
    } else if (eq(f, "__syncwarp")) {
        Str mk = na ? opnd(arg(0)) : S("0xffffffff");
        SB b = sb();
        b.s("    bar.warp.sync ").s(mk).c(';');
        put(b);
    } else if (eq(f, "__activemask")) {
        SB b = sb();
        b.s("    activemask.b32 ").s(dest).c(';');
        put(b);
    } else if (eq(f, "__syncthreads_count") || eq(f, "__syncthreads_and") || eq(f, "__syncthreads_or")) {
        Str src = na ? opnd(arg(0)) : S("0");
        uint32_t pt;
        if (na && arg(0).k == O_VAL && is_pred(vid(arg(0)))) {
            pt = arg(0).x;
        } else {
            pt = new_value(nm("_sp_", dn), S_BOOL);
            add_pred(V(pt).id);
            SB b = sb();
            b.s("    setp.ne.s32 ").s(reg(pt)).s(", ").s(src).s(", 0;");
            put(b);
        }
        if (eq(f, "__syncthreads_count")) {
            SB b = sb();
            b.s("    bar.red.popc.u32 ").s(dest).s(", 0, ").s(reg(pt)).c(';');
            put(b);
        } else {
            uint32_t po = new_value(nm("_sp_out_", dn), S_BOOL);
            add_pred(V(po).id);
            SB b = sb();
            b.s("    bar.red.").s(eq(f, "__syncthreads_and") ? "and" : "or").s(".pred ").s(reg(po)).s(", 0, ").s(reg(pt)).c(';');
            put(b);
            SB b2 = sb();
            b2.s("    selp.s32 ").s(dest).s(", 1, 0, ").s(reg(po)).c(';');
            put(b2);
        }
    } else if (eq(f, "__popc") || eq(f, "__popcll") || eq(f, "__clz") || eq(f, "__clzll") ||
               eq(f, "__brev") || eq(f, "__brevll")) {
        Ty st = na && (arg(0).k == O_VAL || arg(0).k == O_CONST) ? m.opty(arg(0)) : (Ty)S_INT32;
        const char *pt = (!is_ptr(st) && ty_size(st) == 8) ? "b64" : "b32";
        Str src = na ? opnd(arg(0)) : S("0");
        const char *op = sstarts(f, "__popc") ? "popc" : sstarts(f, "__clz") ? "clz" : "brev";
        SB b = sb();
        b.s("    ").s(op).c('.').s(pt).c(' ').s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (eq(f, "__ffs") || eq(f, "__ffsll")) {
        Ty st = na && (arg(0).k == O_VAL || arg(0).k == O_CONST) ? m.opty(arg(0)) : (Ty)S_INT32;
        bool is64 = !is_ptr(st) && ty_size(st) == 8;
        Str src = na ? opnd(arg(0)) : S("0");
        uint32_t tn = new_value(nm("_ffs_neg_", dn), is64 ? S_INT64 : S_INT32);
        uint32_t tl = new_value(nm("_ffs_lsb_", dn), is64 ? S_INT64 : S_INT32);
        uint32_t tp = new_value(nm("_ffs_pos_", dn), S_UINT32);
        SB b = sb();
        b.s("    neg.").s(is64 ? "s64" : "s32").c(' ').s(reg(tn)).s(", ").s(src).c(';');
        put(b);
        SB b2 = sb();
        b2.s("    and.").s(is64 ? "b64" : "b32").c(' ').s(reg(tl)).s(", ").s(src).s(", ").s(reg(tn)).c(';');
        put(b2);
        SB b3 = sb();
        b3.s("    bfind.").s(is64 ? "u64" : "u32").c(' ').s(reg(tp)).s(", ").s(reg(tl)).c(';');
        put(b3);
        SB b4 = sb();
        b4.s("    add.s32 ").s(dest).s(", ").s(reg(tp)).s(", 1;");
        put(b4);
    } else if (a0f64 && in_list(f, " sqrt rsqrt fabs floor ceil trunc round ")) {
        const char *op = eq(f, "sqrt") ? "sqrt.rn.f64" : eq(f, "rsqrt") ? "rsqrt.approx.f64" :
                         eq(f, "fabs") ? "abs.f64" : eq(f, "floor") ? "cvt.rmi.f64.f64" :
                         eq(f, "ceil") ? "cvt.rpi.f64.f64" : eq(f, "trunc") ? "cvt.rzi.f64.f64" :
                         "cvt.rni.f64.f64";
        line1(op, dest, arg0("0d0000000000000000"));
    } else if (a0f64 && in_list(f, " sin cos exp2 log2 ")) {
        const char *op = eq(f, "sin") ? "sin.approx.f32" : eq(f, "cos") ? "cos.approx.f32" :
                         eq(f, "exp2") ? "ex2.approx.f32" : "lg2.approx.f32";
        Str src = arg0("0d0000000000000000");
        uint32_t t32 = new_value(nm("_d2f_", dn), S_FLOAT);
        uint32_t r32 = new_value(nm("_f32r_", dn), S_FLOAT);
        line1("cvt.rn.f32.f64", reg(t32), src);
        line1(op, reg(r32), reg(t32));
        line1("cvt.f64.f32", dest, reg(r32));
    } else if (a0f64 && in_list(f, " exp log log10 exp10 ")) {
        bool lg = eq(f, "log") || eq(f, "log10");
        const char *op = lg ? "lg2.approx.f32" : "ex2.approx.f32";
        const char *sc = eq(f, "exp") ? "0f3FB8AA3B" : eq(f, "log") ? "0f3F317218" :
                         eq(f, "log10") ? "0f3E9A209B" : "0f40549A78";
        Str src = arg0("0d0000000000000000");
        uint32_t t32 = new_value(nm("_d2f_", dn), S_FLOAT);
        uint32_t r32 = new_value(nm("_f32r_", dn), S_FLOAT);
        line1("cvt.rn.f32.f64", reg(t32), src);
        if (lg) {
            uint32_t lo = new_value(nm("_lg2_", dn), S_FLOAT);
            line1(op, reg(lo), reg(t32));
            SB b = sb();
            b.s("    mul.f32 ").s(reg(r32)).s(", ").s(reg(lo)).s(", ").s(sc).c(';');
            put(b);
        } else {
            uint32_t scl = new_value(nm("_scl_", dn), S_FLOAT);
            SB b = sb();
            b.s("    mul.f32 ").s(reg(scl)).s(", ").s(reg(t32)).s(", ").s(sc).c(';');
            put(b);
            line1(op, reg(r32), reg(scl));
        }
        line1("cvt.f64.f32", dest, reg(r32));
    } else if (in_list(f, " expf exp logf log log10f log10 exp10f exp10 ")) {
        bool lg = sstarts(f, "log");
        const char *op = lg ? "lg2.approx.f32" : "ex2.approx.f32";
        const char *sc = (eq(f, "expf") || eq(f, "exp")) ? "0f3FB8AA3B" :
                         (eq(f, "logf") || eq(f, "log")) ? "0f3F317218" :
                         (eq(f, "log10f") || eq(f, "log10")) ? "0f3E9A209B" : "0f40549A78";
        Str src = arg0("0f00000000");
        uint32_t t = new_value(nm("_scale_", dn), S_FLOAT);
        if (lg) {
            line1(op, reg(t), src);
            SB b = sb();
            b.s("    mul.f32 ").s(dest).s(", ").s(reg(t)).s(", ").s(sc).c(';');
            put(b);
        } else {
            SB b = sb();
            b.s("    mul.f32 ").s(reg(t)).s(", ").s(src).s(", ").s(sc).c(';');
            put(b);
            line1(op, dest, reg(t));
        }
    } else if (in_list(f, " sqrtf sqrt rsqrtf rsqrt rcpf sinf sin cosf cos exp2f exp2 log2f log2"
                          " __fsqrt_rn __fsqrt_rd __fsqrt_ru __fsqrt_rz __frcp_rn __frcp_rd"
                          " __frcp_ru __frcp_rz __frsqrt_rn fabsf fabs floorf floor ceilf ceil"
                          " truncf trunc roundf round ")) {
        const char *op =
            (eq(f, "sqrtf") || eq(f, "sqrt")) ? "sqrt.approx.f32" :
            (eq(f, "rsqrtf") || eq(f, "rsqrt") || eq(f, "__frsqrt_rn")) ? "rsqrt.approx.f32" :
            eq(f, "rcpf") ? "rcp.approx.f32" :
            (eq(f, "sinf") || eq(f, "sin")) ? "sin.approx.f32" :
            (eq(f, "cosf") || eq(f, "cos")) ? "cos.approx.f32" :
            (eq(f, "exp2f") || eq(f, "exp2")) ? "ex2.approx.f32" :
            (eq(f, "log2f") || eq(f, "log2")) ? "lg2.approx.f32" :
            eq(f, "__fsqrt_rn") ? "sqrt.rn.f32" : eq(f, "__fsqrt_rd") ? "sqrt.rm.f32" :
            eq(f, "__fsqrt_ru") ? "sqrt.rp.f32" : eq(f, "__fsqrt_rz") ? "sqrt.rz.f32" :
            eq(f, "__frcp_rn") ? "rcp.rn.f32" : eq(f, "__frcp_rd") ? "rcp.rm.f32" :
            eq(f, "__frcp_ru") ? "rcp.rp.f32" : eq(f, "__frcp_rz") ? "rcp.rz.f32" :
            (eq(f, "fabsf") || eq(f, "fabs")) ? "abs.f32" :
            (eq(f, "floorf") || eq(f, "floor")) ? "cvt.rmi.f32.f32" :
            (eq(f, "ceilf") || eq(f, "ceil")) ? "cvt.rpi.f32.f32" :
            (eq(f, "truncf") || eq(f, "trunc")) ? "cvt.rzi.f32.f32" : "cvt.rni.f32.f32";
        line1(op, dest, arg0("0f00000000"));
    } else if (in_list(f, " fminf fmin fmaxf fmax ")) {
        bool mn = eq(f, "fminf") || eq(f, "fmin");
        const char *op = a0f64 ? (mn ? "min.f64" : "max.f64") : (mn ? "min.f32" : "max.f32");
        Str a = arg0("0f00000000");
        Str bb = na > 1 ? opnd(arg(1)) : S("0f00000000");
        SB b = sb();
        b.s("    ").s(op).c(' ').s(dest).s(", ").s(a).s(", ").s(bb).c(';');
        put(b);
    } else if (in_list(f, " fmaf fma __fmaf_rn __fmaf_rd __fmaf_ru __fmaf_rz __fma_rn __fma_rd"
                          " __fma_ru __fma_rz ")) {
        const char *ft = a0f64 ? "f64" : "f32";
        char rnd[3] = {'r', 'n', 0};
        if (f.n >= 2) {
            char x0 = f.p[f.n - 2], x1 = f.p[f.n - 1];
            if (x0 == 'r' && (x1 == 'n' || x1 == 'd' || x1 == 'u' || x1 == 'z')) rnd[1] = x1;
        }
        Str a = arg0("0f00000000");
        Str bb = na > 1 ? opnd(arg(1)) : S("0f00000000");
        Str c = na > 2 ? opnd(arg(2)) : S("0f00000000");
        SB b = sb();
        b.s("    fma.").s(rnd).c('.').s(ft).c(' ').s(dest).s(", ").s(a).s(", ").s(bb).s(", ").s(c).c(';');
        put(b);
    } else if (eq(f, "fmodf") || eq(f, "fmod")) {
        Str x = arg0("0f00000000");
        Str y = na > 1 ? opnd(arg(1)) : S("0f00000000");
        uint32_t q = new_value(nm("_fmod_q_", dn), S_FLOAT);
        uint32_t qt = new_value(nm("_fmod_qt_", dn), S_FLOAT);
        uint32_t qy = new_value(nm("_fmod_qy_", dn), S_FLOAT);
        SB b = sb();
        b.s("    div.approx.f32 ").s(reg(q)).s(", ").s(x).s(", ").s(y).c(';');
        put(b);
        line1("cvt.rzi.f32.f32", reg(qt), reg(q));
        SB b2 = sb();
        b2.s("    mul.f32 ").s(reg(qy)).s(", ").s(reg(qt)).s(", ").s(y).c(';');
        put(b2);
        SB b3 = sb();
        b3.s("    sub.f32 ").s(dest).s(", ").s(x).s(", ").s(reg(qy)).c(';');
        put(b3);
    } else if (eq(f, "tanf") || eq(f, "tan")) {
        Str x = arg0("0f00000000");
        uint32_t s_ = new_value(nm("_tan_s_", dn), S_FLOAT);
        uint32_t c = new_value(nm("_tan_c_", dn), S_FLOAT);
        line1("sin.approx.f32", reg(s_), x);
        line1("cos.approx.f32", reg(c), x);
        SB b = sb();
        b.s("    div.approx.f32 ").s(dest).s(", ").s(reg(s_)).s(", ").s(reg(c)).c(';');
        put(b);
    } else if (eq(f, "abs")) {
        Ty ty = in.dest >= 0 ? V((uint32_t)in.dest).ty : (Ty)S_INT32;
        SB op = sb();
        op.s("abs.").s(ptx_type(ty));
        Str src = na ? opnd(arg(0)) : S("0");
        SB b = sb();
        b.s("    ").s(op.str()).c(' ').s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (eq(f, "min") || eq(f, "max")) {
        Ty ty = in.dest >= 0 ? V((uint32_t)in.dest).ty : (Ty)S_INT32;
        const char *pt = ptx_type(ty);
        Str a = na ? opnd(arg(0), pt) : S("0");
        Str bb = na > 1 ? opnd(arg(1), pt) : S("0");
        SB b = sb();
        b.s("    ").s(eq(f, "min") ? "min" : "max").c('.').s(pt).c(' ').s(dest).s(", ").s(a).s(", ").s(bb).c(';');
        put(b);
    } else if (in_list(f, " isnan isinf isfinite __isnan __isinf __isfinite __isnanf __isinff __isfinitef ")) {
        const char *prop = contains(f, "nan") ? "notanumber" : contains(f, "inf") ? "infinite" : "finite";
        if (contains(f, "finite")) prop = "finite";
        Ty st = na && (arg(0).k == O_VAL || arg(0).k == O_CONST) ? m.opty(arg(0)) : (Ty)S_FLOAT;
        const char *ft = (!is_ptr(st) && ty_size(st) == 8) ? "f64" : "f32";
        Str src = arg0("0f00000000");
        uint32_t pt = new_value(nm("_tp_", dn), S_BOOL);
        add_pred(V(pt).id);
        SB b = sb();
        b.s("    testp.").s(prop).c('.').s(ft).c(' ').s(reg(pt)).s(", ").s(src).c(';');
        put(b);
        SB b2 = sb();
        b2.s("    selp.s32 ").s(dest).s(", 1, 0, ").s(reg(pt)).c(';');
        put(b2);
    } else if (sstarts(f, "__float2int_") || sstarts(f, "__float2uint_") || sstarts(f, "__float2ll_") ||
               sstarts(f, "__float2ull_")) {
        if (!in_list(f, kFloat2Int)) { unsup(); return; }
        char last = f.p[f.n - 1];
        const char *rnd = last == 'n' ? "rni" : last == 'd' ? "rmi" : last == 'u' ? "rpi" : "rzi";
        const char *it = sstarts(f, "__float2int_") ? "s32" : sstarts(f, "__float2uint_") ? "u32" :
                         sstarts(f, "__float2ll_") ? "s64" : "u64";
        Str src = arg0("0f00000000");
        SB b = sb();
        b.s("    cvt.").s(rnd).c('.').s(it).s(".f32 ").s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (in_list(f, " __double2int_rn __double2int_rz __double2uint_rn __double2uint_rz"
                          " __double2ll_rn __double2ll_rz __double2ull_rn __double2ull_rz ")) {
        const char *rnd = f.p[f.n - 1] == 'n' ? "rni" : "rzi";
        const char *it = sstarts(f, "__double2int_") ? "s32" : sstarts(f, "__double2uint_") ? "u32" :
                         sstarts(f, "__double2ll_") ? "s64" : "u64";
        Str src = arg0("0d0000000000000000");
        SB b = sb();
        b.s("    cvt.").s(rnd).c('.').s(it).s(".f64 ").s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (in_list(f, " __int2float_rn __int2float_rd __int2float_ru __int2float_rz"
                          " __uint2float_rn __uint2float_rd __uint2float_ru __uint2float_rz"
                          " __ll2float_rn __ll2float_rz __ull2float_rn __ull2float_rz ")) {
        char last = f.p[f.n - 1];
        const char *rnd = last == 'n' ? "rn" : last == 'd' ? "rm" : last == 'u' ? "rp" : "rz";
        const char *it = sstarts(f, "__int2") ? "s32" : sstarts(f, "__uint2") ? "u32" :
                         sstarts(f, "__ll2") ? "s64" : "u64";
        Str src = arg0("0");
        SB b = sb();
        b.s("    cvt.").s(rnd).s(".f32.").s(it).c(' ').s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (in_list(f, " __int2double_rn __ll2double_rn __uint2double_rn __ull2double_rn ")) {
        const char *it = contains(f, "ull") ? "u64" : contains(f, "ll") ? "s64" :
                         contains(f, "uint") ? "u32" : "s32";
        Str src = arg0("0");
        SB b = sb();
        b.s("    cvt.rn.f64.").s(it).c(' ').s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (in_list(f, " __float_as_int __float_as_uint ")) {
        line1("mov.b32", dest, arg0("0f00000000"));
    } else if (in_list(f, " __int_as_float __uint_as_float ")) {
        line1("mov.b32", dest, arg0("0"));
    } else if (in_list(f, " __double_as_longlong __double_as_ulonglong ")) {
        line1("mov.b64", dest, arg0("0d0000000000000000"));
    } else if (in_list(f, " __longlong_as_double __ulonglong_as_double ")) {
        line1("mov.b64", dest, arg0("0"));
    } else if (eq(f, "__sad") || eq(f, "__usad")) {
        Str a = arg0("0");
        Str bb = na > 1 ? opnd(arg(1)) : S("0");
        Str c = na > 2 ? opnd(arg(2)) : S("0");
        SB b = sb();
        b.s("    sad.").s(eq(f, "__usad") ? "u32" : "s32").c(' ').s(dest).s(", ").s(a).s(", ").s(bb).s(", ").s(c).c(';');
        put(b);
    } else if (eq(f, "warpSize")) {
        SB b = sb();
        b.s("    mov.u32 ").s(dest).s(", 32;");
        put(b);
    } else if (in_list(f, " __mul24 __umul24 __mulhi __umulhi ")) {
        // integer multiplies (emit.py:2493-2508)
        const char *op = eq(f, "__mul24") ? "mul24.lo.s32" : eq(f, "__umul24") ? "mul24.lo.u32" :
                         eq(f, "__mulhi") ? "mul.hi.s32" : "mul.hi.u32";
        Str a = arg0("0");
        Str bb = na > 1 ? opnd(arg(1)) : S("0");
        SB b = sb();
        b.s("    ").s(op).c(' ').s(dest).s(", ").s(a).s(", ").s(bb).c(';');
        put(b);
    } else if (sstarts(f, "__reduce_") && in_list(f, " __reduce_add_sync __reduce_min_sync __reduce_max_sync "
                   "__reduce_and_sync __reduce_or_sync __reduce_xor_sync __reduce_umin_sync __reduce_umax_sync ")) {
        // redux.sync (emit.py:2447-2479): value first, mask second in the instruction
        const char *op = eq(f, "__reduce_add_sync") ? "add.s32" : eq(f, "__reduce_min_sync") ? "min.s32" :
                         eq(f, "__reduce_max_sync") ? "max.s32" : eq(f, "__reduce_and_sync") ? "and.b32" :
                         eq(f, "__reduce_or_sync") ? "or.b32" : eq(f, "__reduce_xor_sync") ? "xor.b32" :
                         eq(f, "__reduce_umin_sync") ? "min.u32" : "max.u32";
        Str mk = arg0("0xffffffff");
        Str val = na > 1 ? opnd(arg(1)) : S("0");
        SB b = sb();
        b.s("    redux.sync.").s(op).c(' ').s(dest).s(", ").s(val).s(", ").s(mk).c(';');
        put(b);
    } else if (eq(f, "__match_any_sync") || eq(f, "__match_all_sync")) {  // emit.py:2480-2491
        Str mk = arg0("0xffffffff");
        Str val = na > 1 ? opnd(arg(1)) : S("0");
        SB b = sb();
        b.s("    match.").s(eq(f, "__match_any_sync") ? "any" : "all").s(".sync.b32 ").s(dest).s(", ").s(val)
            .s(", ").s(mk).c(';');
        put(b);
    } else if (in_list(f, " __hadd __hadd_rn __hadd_sat ")) {  // emit.py:2509-2523
        Ty dty = in.dest >= 0 ? V((uint32_t)in.dest).ty : (Ty)S_INT32;
        if (!is_ptr(dty) && ty_scalar(dty) == S_HALF) {  // f16 add
            Str a = arg0("0h0000");
            Str bb = na > 1 ? opnd(arg(1)) : S("0h0000");
            SB b = sb();
            b.s("    add.rn").s(eq(f, "__hadd_sat") ? ".sat" : "").s(".f16 ").s(dest).s(", ").s(a).s(", ").s(bb).c(';');
            put(b);
        } else {  // integer halving add: (a + b) >> 1
            Str a = arg0("0");
            Str bb = na > 1 ? opnd(arg(1)) : S("0");
            uint32_t t = new_value(nm("_hadd_tmp_", dn), S_INT32);
            SB b1 = sb();
            b1.s("    add.s32 ").s(reg(t)).s(", ").s(a).s(", ").s(bb).c(';');
            put(b1);
            SB b2 = sb();
            b2.s("    shr.s32 ").s(dest).s(", ").s(reg(t)).s(", 1;");
            put(b2);
        }
    } else if (eq(f, "__rhadd")) {  // (a + b + 1) >> 1 unsigned (emit.py:2524-2532)
        Str a = arg0("0");
        Str bb = na > 1 ? opnd(arg(1)) : S("0");
        uint32_t t = new_value(nm("_rhadd_tmp_", dn), S_UINT32);
        SB b1 = sb();
        b1.s("    add.u32 ").s(reg(t)).s(", ").s(a).s(", ").s(bb).c(';');
        put(b1);
        SB b2 = sb();
        b2.s("    add.u32 ").s(reg(t)).s(", ").s(reg(t)).s(", 1;");
        put(b2);
        SB b3 = sb();
        b3.s("    shr.u32 ").s(dest).s(", ").s(reg(t)).s(", 1;");
        put(b3);
    } else if (eq(f, "__ushort_as_half") || eq(f, "__short_as_half")) {  // emit.py:2554-2569
        SB b = sb();
        if (!na) {
            b.s("    mov.b16 ").s(dest).s(", 0;");
        } else {
            Str src = opnd(arg(0));
            if (sstarts(src, "%r")) {  // low half of a b32 register by vector unpack
                uint32_t dc = new_value(nm("_half_discard_", dn), S_HALF);
                b.s("    mov.b32 {").s(dest).s(", ").s(reg(dc)).s("}, ").s(src).c(';');
            } else {
                b.s("    mov.b16 ").s(dest).s(", ").s(src).c(';');
            }
        }
        put(b);
    } else if (eq(f, "__half_as_ushort") || eq(f, "__half_as_short")) {  // emit.py:2570-2585
        if (!na) {
            SB b = sb();
            b.s("    mov.b32 ").s(dest).s(", 0;");
            put(b);
        } else {
            Str src = opnd(arg(0));
            if (sstarts(src, "%h")) {  // pack with a zero half
                uint32_t z = new_value(nm("_half_zero_", dn), S_HALF);
                SB b1 = sb();
                b1.s("    mov.b16 ").s(reg(z)).s(", 0;");
                put(b1);
                SB b2 = sb();
                b2.s("    mov.b32 ").s(dest).s(", {").s(src).s(", ").s(reg(z)).s("};");
                put(b2);
            } else {
                SB b = sb();
                b.s("    mov.b16 ").s(dest).s(", ").s(src).c(';');
                put(b);
            }
        }
    } else if (in_list(f, " __int2half_rn __uint2half_rn __short2half_rn __ushort2half_rn __ll2half_rn __ull2half_rn "
                          "__int2half_rz __uint2half_rz __ll2half_rz __ull2half_rz ")) {  // emit.py:2586-2600
        Str src = arg0("0");
        const char *sp = na && arg(0).k == O_VAL ? ptx_type(V(arg(0).x).ty) : "s32";
        SB b = sb();
        b.s("    cvt.").s(ends_with(f, "_rz") ? "rz" : "rn").s(".f16.").s(sp).c(' ').s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (in_list(f, " __half2int_rn __half2uint_rn __half2short_rn __half2ushort_rn __half2ll_rn __half2ull_rn "
                          "__half2int_rz __half2uint_rz __half2short_rz __half2ushort_rz __half2ll_rz __half2ull_rz ")) {
        // emit.py:2601-2614
        Str src = arg0("0h0000");
        const char *dp = in.dest >= 0 ? ptx_type(V((uint32_t)in.dest).ty) : "s32";
        SB b = sb();
        b.s("    cvt.").s(ends_with(f, "_rz") ? "rzi." : "rni.").s(dp).s(".f16 ").s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (in_list(f, " __float2half __float2half_rn __float2half_rd __float2half_ru __float2half_rz ")) {
        // emit.py:2615-2626
        const char *rm = eq(f, "__float2half_rd") ? "rm" : eq(f, "__float2half_ru") ? "rp" :
                         eq(f, "__float2half_rz") ? "rz" : "rn";
        Str src = arg0("0f00000000");
        SB b = sb();
        b.s("    cvt.").s(rm).s(".f16.f32 ").s(dest).s(", ").s(src).c(';');
        put(b);
    } else if (in_list(f, " __half2float __low2float __high2float ")) {  // emit.py:2627-2629
        line1("cvt.f32.f16", dest, arg0("0h0000"));
    } else if (in_list(f, " __hmul __hmul_rn __hmul_sat __hsub __hsub_rn __hfmin __hmin __hfmax __hmax ")) {
        // two-operand f16 arithmetic (emit.py:2630-2641, 2655-2662)
        const char *op = eq(f, "__hmul_sat") ? "mul.rn.sat.f16" : sstarts(f, "__hmul") ? "mul.rn.f16" :
                         sstarts(f, "__hsub") ? "sub.rn.f16" : (eq(f, "__hfmin") || eq(f, "__hmin")) ? "min.f16" :
                         "max.f16";
        Str a = arg0("0h0000");
        Str bb = na > 1 ? opnd(arg(1)) : S("0h0000");
        SB b = sb();
        b.s("    ").s(op).c(' ').s(dest).s(", ").s(a).s(", ").s(bb).c(';');
        put(b);
    } else if (in_list(f, " __hfma __hfma_sat __hfma_relu ")) {  // emit.py:2663-2673
        Str a = arg0("0h0000");
        Str bb = na > 1 ? opnd(arg(1)) : S("0h0000");
        Str c = na > 2 ? opnd(arg(2)) : S("0h0000");
        SB b = sb();
        b.s("    fma.rn").s(eq(f, "__hfma_sat") ? ".sat" : eq(f, "__hfma_relu") ? ".relu" : "").s(".f16 ").s(dest)
            .s(", ").s(a).s(", ").s(bb).s(", ").s(c).c(';');
        put(b);
    } else if (eq(f, "__habs") || eq(f, "__hneg")) {  // emit.py:2674-2679
        line1(eq(f, "__habs") ? "abs.f16" : "neg.f16", dest, arg0("0h0000"));
    } else if (eq(f, "__hexp2")) {  // emit.py:2722-2725
        line1("ex2.approx.f16", dest, arg0("0h0000"));
    } else if (eq(f, "__hdiv")) {  // a * f16(rcp(f32(b))) (emit.py:2642-2654)
        Str a = arg0("0h0000");
        Str bb = na > 1 ? opnd(arg(1)) : S("0h3C00");
        uint32_t fb = new_value(nm("_hdiv_b_", dn), S_FLOAT);
        uint32_t fr = new_value(nm("_hdiv_r_", dn), S_FLOAT);
        uint32_t hr = new_value(nm("_hdiv_h_", dn), S_HALF);
        line1("cvt.f32.f16", reg(fb), bb);
        line1("rcp.approx.f32", reg(fr), reg(fb));
        line1("cvt.rn.f16.f32", reg(hr), reg(fr));
        SB b = sb();
        b.s("    mul.rn.f16 ").s(dest).s(", ").s(a).s(", ").s(reg(hr)).c(';');
        put(b);
    } else if (in_list(f, " __hrcp __hsqrt __hrsqrt __hexp __hlog __hceil __hfloor __hrint __htrunc "
                          "__hcos __hsin __hlog2 __hlog10 ")) {
        // through f32 and back (emit.py:2680-2721)
        Str src = arg0("0h0000");
        uint32_t fi = new_value(nm("_hf32in_", dn), S_FLOAT);
        uint32_t fo = new_value(nm("_hf32out_", dn), S_FLOAT);
        line1("cvt.f32.f16", reg(fi), src);
        if (eq(f, "__hrcp")) {
            line1("rcp.approx.f32", reg(fo), reg(fi));
        } else if (eq(f, "__hsqrt")) {
            line1("sqrt.approx.f32", reg(fo), reg(fi));
        } else if (eq(f, "__hrsqrt")) {
            line1("rsqrt.approx.f32", reg(fo), reg(fi));
        } else if (eq(f, "__hexp")) {
            uint32_t sc = new_value(nm("_hscale_", dn), S_FLOAT);
            SB b = sb();
            b.s("    mul.f32 ").s(reg(sc)).s(", ").s(reg(fi)).s(", 0f3FB8AA3B;");
            put(b);
            line1("ex2.approx.f32", reg(fo), reg(sc));
        } else if (eq(f, "__hlog") || eq(f, "__hlog10")) {
            uint32_t lg = new_value(nm("_hlg2_", dn), S_FLOAT);
            line1("lg2.approx.f32", reg(lg), reg(fi));
            SB b = sb();
            b.s("    mul.f32 ").s(reg(fo)).s(", ").s(reg(lg)).s(eq(f, "__hlog") ? ", 0f3F317218;" : ", 0f3E9A209B;");
            put(b);
        } else if (eq(f, "__hlog2")) {
            line1("lg2.approx.f32", reg(fo), reg(fi));
        } else if (eq(f, "__hcos")) {
            line1("cos.approx.f32", reg(fo), reg(fi));
        } else if (eq(f, "__hsin")) {
            line1("sin.approx.f32", reg(fo), reg(fi));
        } else {
            uint32_t it = new_value(nm("_hint_", dn), S_INT32);
            const char *rm = eq(f, "__hceil") ? "cvt.rpi.s32.f32" : eq(f, "__hfloor") ? "cvt.rmi.s32.f32" :
                             eq(f, "__hrint") ? "cvt.rni.s32.f32" : "cvt.rzi.s32.f32";
            line1(rm, reg(it), reg(fi));
            line1("cvt.rn.f32.s32", reg(fo), reg(it));
        }
        line1("cvt.rn.f16.f32", dest, reg(fo));
    } else if (in_list(f, " __hgt __hlt __hge __hle __heq __hne ")) {  // setp.f16 + selp (emit.py:2726-2738)
        const char *cmp = eq(f, "__hgt") ? "gt" : eq(f, "__hlt") ? "lt" : eq(f, "__hge") ? "ge" :
                          eq(f, "__hle") ? "le" : eq(f, "__heq") ? "eq" : "ne";
        Str a = arg0("0h0000");
        Str bb = na > 1 ? opnd(arg(1)) : S("0h0000");
        uint32_t pt = new_value(nm("_hcmp_", dn), S_BOOL);
        add_pred(V(pt).id);
        SB b1 = sb();
        b1.s("    setp.").s(cmp).s(".f16 ").s(reg(pt)).s(", ").s(a).s(", ").s(bb).c(';');
        put(b1);
        SB b2 = sb();
        b2.s("    selp.s32 ").s(dest).s(", 1, 0, ").s(reg(pt)).c(';');
        put(b2);
    } else if (eq(f, "__hisnan") || eq(f, "__hisinf")) {  // via f32 testp (emit.py:2739-2749)
        Str src = arg0("0h0000");
        uint32_t ft = new_value(nm("_h2f_", dn), S_FLOAT);
        uint32_t pt = new_value(nm("_htest_", dn), S_BOOL);
        add_pred(V(pt).id);
        line1("cvt.f32.f16", reg(ft), src);
        SB b1 = sb();
        b1.s("    testp.").s(eq(f, "__hisnan") ? "notanumber" : "infinite").s(".f32 ").s(reg(pt)).s(", ")
            .s(reg(ft)).c(';');
        put(b1);
        SB b2 = sb();
        b2.s("    selp.s32 ").s(dest).s(", 1, 0, ").s(reg(pt)).c(';');
        put(b2);
    } else if (in_list(f, " asinf asin acosf acos ")) {
        // asin(x) = atan(x / sqrt(1 - x^2)) with the atan series; acos = pi/2 - asin (emit.py:2772-2829)
        bool ac = sstarts(f, "acos");
        const char *pf = ac ? "_acos_" : "_asin_";
        Str x = arg0("0f00000000");
        auto val = [&](const char *suffix) {
            SB b = sb();
            b.s(pf).s(suffix).i(dn);
            return new_value(b.str(), S_FLOAT);
        };
        uint32_t x2 = val("x2_"), om = val("om_"), sq = val("sq_"), rat = val("r_");
        uint32_t ax2 = val("ax2_"), ax4 = val("ax4_"), ax6 = val("ax6_"), pp = val("p_"), p2 = val("p2_");
        uint32_t as = ac ? val("as_") : 0;
        SB b1 = sb();
        b1.s("    mul.f32 ").s(reg(x2)).s(", ").s(x).s(", ").s(x).c(';');
        put(b1);
        SB b2 = sb();
        b2.s("    fma.rn.f32 ").s(reg(om)).s(", ").s(reg(x2)).s(", 0fBF800000, 0f3F800000;");
        put(b2);
        line1("sqrt.approx.f32", reg(sq), reg(om));
        SB b3 = sb();
        b3.s("    div.approx.f32 ").s(reg(rat)).s(", ").s(x).s(", ").s(reg(sq)).c(';');
        put(b3);
        SB b4 = sb();
        b4.s("    mul.f32 ").s(reg(ax2)).s(", ").s(reg(rat)).s(", ").s(reg(rat)).c(';');
        put(b4);
        SB b5 = sb();
        b5.s("    mul.f32 ").s(reg(ax4)).s(", ").s(reg(ax2)).s(", ").s(reg(ax2)).c(';');
        put(b5);
        SB b6 = sb();
        b6.s("    mul.f32 ").s(reg(ax6)).s(", ").s(reg(ax4)).s(", ").s(reg(ax2)).c(';');
        put(b6);
        SB b7 = sb();
        b7.s("    fma.rn.f32 ").s(reg(pp)).s(", ").s(reg(ax6)).s(", 0fBE124925, 0f3F800000;");
        put(b7);
        SB b8 = sb();
        b8.s("    fma.rn.f32 ").s(reg(p2)).s(", ").s(reg(ax4)).s(", 0f3E4CCCCD, ").s(reg(pp)).c(';');
        put(b8);
        SB b9 = sb();
        b9.s("    fma.rn.f32 ").s(reg(pp)).s(", ").s(reg(ax2)).s(", 0fBEAAAAAB, ").s(reg(p2)).c(';');
        put(b9);
        SB b10 = sb();
        b10.s("    mul.f32 ").s(ac ? reg(as) : dest).s(", ").s(reg(rat)).s(", ").s(reg(pp)).c(';');
        put(b10);
        if (ac) {
            SB b11 = sb();
            b11.s("    sub.f32 ").s(dest).s(", 0f3FC90FDB, ").s(reg(as)).c(';');
            put(b11);
        }
    } else if (in_list(f, " __dp4a __dp4a_u __dp4a_su __dp4a_us ")) {  // emit.py:2433-2446
        const char *op = eq(f, "__dp4a_u") ? "dp4a.u32.u32" : eq(f, "__dp4a_su") ? "dp4a.s32.u32" :
                         eq(f, "__dp4a_us") ? "dp4a.u32.s32" : "dp4a.s32.s32";
        Str a = arg0("0");
        Str bb = na > 1 ? opnd(arg(1)) : S("0");
        Str c = na > 2 ? opnd(arg(2)) : S("0");
        SB b = sb();
        b.s("    ").s(op).c(' ').s(dest).s(", ").s(a).s(", ").s(bb).s(", ").s(c).c(';');
        put(b);
    } else if (in_list(f, " __funnelshift_l __funnelshift_lc __funnelshift_r __funnelshift_rc ")) {
        // shf (emit.py:2540-2553): clamp for the *c forms, wrap otherwise
        Str lo = arg0("0");
        Str hi = na > 1 ? opnd(arg(1)) : S("0");
        Str sh = na > 2 ? opnd(arg(2)) : S("0");
        bool left = sstarts(f, "__funnelshift_l");
        bool clamp = f.p[f.n - 1] == 'c';
        SB b = sb();
        b.s("    shf.").s(left ? "l" : "r").c('.').s(clamp ? "clamp" : "wrap").s(".b32 ").s(dest)
            .s(", ").s(lo).s(", ").s(hi).s(", ").s(sh).c(';');
        put(b);
    } else if (in_list(f, " atanf atan ")) {  // x * (1 - x^2/3 + x^4/5 - x^6/7) (emit.py:2756-2771)
        Str x = arg0("0f00000000");
        uint32_t x2 = new_value(nm("_atan_x2_", dn), S_FLOAT);
        uint32_t x4 = new_value(nm("_atan_x4_", dn), S_FLOAT);
        uint32_t x6 = new_value(nm("_atan_x6_", dn), S_FLOAT);
        uint32_t pp = new_value(nm("_atan_p_", dn), S_FLOAT);
        uint32_t p2 = new_value(nm("_atan_p2_", dn), S_FLOAT);
        SB b1 = sb();
        b1.s("    mul.f32 ").s(reg(x2)).s(", ").s(x).s(", ").s(x).c(';');
        put(b1);
        SB b2 = sb();
        b2.s("    mul.f32 ").s(reg(x4)).s(", ").s(reg(x2)).s(", ").s(reg(x2)).c(';');
        put(b2);
        SB b3 = sb();
        b3.s("    mul.f32 ").s(reg(x6)).s(", ").s(reg(x4)).s(", ").s(reg(x2)).c(';');
        put(b3);
        SB b4 = sb();
        b4.s("    fma.rn.f32 ").s(reg(pp)).s(", ").s(reg(x6)).s(", 0fBE124925, 0f3F800000;");
        put(b4);
        SB b5 = sb();
        b5.s("    fma.rn.f32 ").s(reg(p2)).s(", ").s(reg(x4)).s(", 0f3E4CCCCD, ").s(reg(pp)).c(';');
        put(b5);
        SB b6 = sb();
        b6.s("    fma.rn.f32 ").s(reg(pp)).s(", ").s(reg(x2)).s(", 0fBEAAAAAB, ").s(reg(p2)).c(';');
        put(b6);
        SB b7 = sb();
        b7.s("    mul.f32 ").s(dest).s(", ").s(x).s(", ").s(reg(pp)).c(';');
        put(b7);
    } else if (in_list(f, " atan2f atan2 ")) {  // y/x through a truncated series (emit.py:2854-2885)
        Str y = arg0("0f00000000");
        Str x = na > 1 ? opnd(arg(1)) : S("0f3F800000");
        uint32_t ratio = new_value(nm("_atan2_r_", dn), S_FLOAT);
        new_value(nm("_atan2_l_", dn), S_FLOAT);   // allocated but unused, as there
        new_value(nm("_atan2_e_", dn), S_FLOAT);
        new_value(nm("_atan2_sv_", dn), S_FLOAT);
        new_value(nm("_atan2_cv_", dn), S_FLOAT);
        uint32_t t2 = new_value(nm("_atan2_t2_", dn), S_FLOAT);
        uint32_t t4 = new_value(nm("_atan2_t4_", dn), S_FLOAT);
        uint32_t poly = new_value(nm("_atan2_p_", dn), S_FLOAT);
        SB b1 = sb();
        b1.s("    div.approx.f32 ").s(reg(ratio)).s(", ").s(y).s(", ").s(x).c(';');
        put(b1);
        SB b2 = sb();
        b2.s("    mul.f32 ").s(reg(t2)).s(", ").s(reg(ratio)).s(", ").s(reg(ratio)).c(';');
        put(b2);
        SB b3 = sb();
        b3.s("    mul.f32 ").s(reg(t4)).s(", ").s(reg(t2)).s(", ").s(reg(t2)).c(';');
        put(b3);
        SB b4 = sb();
        b4.s("    fma.rn.f32 ").s(reg(poly)).s(", ").s(reg(t4)).s(", 0f3E4CCCCD, ").s(reg(ratio)).c(';');
        put(b4);
        SB b5 = sb();
        b5.s("    fma.rn.f32 ").s(dest).s(", ").s(reg(t2)).s(", 0fBEAAAAAB, ").s(reg(poly)).c(';');
        put(b5);
    } else if (eq(f, "__byte_perm")) {  // prmt (emit.py:2534-2539)
        Str a = arg0("0");
        Str bb = na > 1 ? opnd(arg(1)) : S("0");
        Str sel = na > 2 ? opnd(arg(2)) : S("0");
        SB b = sb();
        b.s("    prmt.b32 ").s(dest).s(", ").s(a).s(", ").s(bb).s(", ").s(sel).c(';');
        put(b);
    } else if (in_list(f, " powf pow ")) {  // exp2(y * log2(x)) (emit.py:2824-2833)
        Str x = arg0("0f00000000");
        Str y = na > 1 ? opnd(arg(1)) : S("0f3F800000");
        uint32_t lg = new_value(nm("_pow_lg2x_", dn), S_FLOAT);
        uint32_t yl = new_value(nm("_pow_ylg2x_", dn), S_FLOAT);
        line1("lg2.approx.f32", reg(lg), x);
        SB b = sb();
        b.s("    mul.f32 ").s(reg(yl)).s(", ").s(y).s(", ").s(reg(lg)).c(';');
        put(b);
        line1("ex2.approx.f32", dest, reg(yl));
    } else if (in_list(f, " hypotf hypot ")) {  // sqrt(a*a + b*b) (emit.py:2834-2843)
        Str a = arg0("0f00000000");
        Str bb = na > 1 ? opnd(arg(1)) : S("0f00000000");
        uint32_t a2 = new_value(nm("_hypot_a2_", dn), S_FLOAT);
        uint32_t ab = new_value(nm("_hypot_ab2_", dn), S_FLOAT);
        SB b = sb();
        b.s("    mul.f32 ").s(reg(a2)).s(", ").s(a).s(", ").s(a).c(';');
        put(b);
        SB b2 = sb();
        b2.s("    fma.rn.f32 ").s(reg(ab)).s(", ").s(bb).s(", ").s(bb).s(", ").s(reg(a2)).c(';');
        put(b2);
        line1("sqrt.approx.f32", dest, reg(ab));
    } else if (in_list(f, " cbrtf cbrt ")) {  // exp2(log2(x) / 3) (emit.py:2844-2853)
        Str x = arg0("0f00000000");
        uint32_t lg = new_value(nm("_cbrt_lg2x_", dn), S_FLOAT);
        uint32_t l3 = new_value(nm("_cbrt_lg2x3_", dn), S_FLOAT);
        line1("lg2.approx.f32", reg(lg), x);
        SB b = sb();
        b.s("    mul.f32 ").s(reg(l3)).s(", ").s(reg(lg)).s(", 0f3EAAAAAB;");
        put(b);
        line1("ex2.approx.f32", dest, reg(l3));
    } else if (in_list(f, ref_call_names()) || sstarts(f, "atomic") || sstarts(f, "__devfn_")) {
        unsup();  // other intrinsics the reference expands (half, dp4a, warp reductions, atan2, ...)
    }
    // any other name: the reference emits nothing for the call
}

OCB_HD inline void Emit::emit_inst(uint32_t ix) {
    const Inst in = I(ix);
    switch (in.kind) {
    case I_PARAM: {
        Ty ty = V((uint32_t)in.dest).ty;
        const char *pt = ptx_type(ty);
        if (cstr_eq(pt, "f16")) pt = "b16";
        SB b = sb();
        b.s("    ld.param.").s(pt).c(' ').s(reg(in.dest)).s(", [").s(in.func).s("];");
        put(b);
        break;
    }
    case I_GADDR: {  // generic address of the symbol, then into its state space (emit.py:1169-1178)
        Str d = reg(in.dest);
        SB b1 = sb();
        b1.s("    mov.u64 ").s(d).s(", ").s(in.func).c(';');
        put(b1);
        SB b2 = sb();
        b2.s("    cvta.to.").s(in.op == AS_CONST ? "const" : "global").s(".u64 ").s(d).s(", ").s(d).c(';');
        put(b2);
        break;
    }
    case I_BIN: emit_bin(in); break;
    case I_CMP: emit_cmp(in); break;
    case I_CVT: emit_cvt(in); break;
    case I_LOAD: emit_load(in); break;
    case I_STORE: emit_store(in); break;
    case I_CALL: emit_call(in); break;
    case I_PRINTF: emit_printf(in); break;
    case I_ASM: emit_asm(in); break;
    default: unsup(); break;
    }
}

// printf -> vprintf (emit.py:1661-1740): the format string's address, the
// arguments widened to 8-byte slots of a .local buffer (f32 to f64, 32-bit
// integers sign- or zero-extended), its generic address, and the call.
OCB_HD inline void Emit::emit_printf(const Inst &in) {
    if (pf_idx >= pfs.n) return;
    Str label = pfs[pf_idx++].label;
    uint32_t nargs = in.args.n;
    uint32_t n = pf_count++;
    bool ok = true;
    Ty gptr = ty_ptr(S_VOID, AS_GLOBAL, false, ok);
    Ty lptr = ty_ptr(S_VOID, AS_LOCAL, false, ok);
    Ty vptr = ty_ptr(S_VOID, AS_GENERIC, false, ok);
    uint32_t fa = new_value(nm("_fmt_addr_", n), gptr);
    {
        Str r = reg(fa);
        SB b = sb();
        b.s("    mov.u64 ").s(r).s(", ").s(label).c(';');
        put(b);
    }
    Str va;
    if (nargs > 0) {
        uint32_t vl = new_value(nm("_valist_", n), lptr);
        {
            SB b = sb();
            b.s("    .local .align 8 .b8 _valist_").i(n).c('[').i(8 * (pyint)nargs).s("];");
            put(b);
            Str r = reg(vl);
            SB b2 = sb();
            b2.s("    mov.u64 ").s(r).s(", _valist_").i(n).c(';');
            put(b2);
        }
        for (uint32_t i = 0; i < nargs && !bad(); ++i) {
            Opnd a = in.args[i];
            Ty at = (a.k == O_VAL || a.k == O_CONST) ? m.opty(a) : (Ty)S_INT32;
            bool fl = ty_is_scalar(at) && ty_is_float(at);
            bool w64 = is_ptr(at) || (ty_is_scalar(at) && ty_size(at) == 8);
            Str sv;
            const char *sty;
            if (fl && !w64) {
                uint32_t pr = new_value(nm2("_va_arg_", n, "_", i), S_DOUBLE);
                Str r = reg(pr);
                Str o = opnd(a);
                SB b = sb();
                b.s("    cvt.f64.f32 ").s(r).s(", ").s(o).c(';');
                put(b);
                sv = r;
                sty = "f64";
            } else if (!w64 && !fl) {
                uint32_t wv = new_value(nm2("_va_arg_", n, "_", i), gptr);
                Str r = reg(wv);
                Str o = opnd(a);
                SB b = sb();
                b.s(ty_is_scalar(at) && ty_is_signed(at) ? "    cvt.s64.s32 " : "    cvt.u64.u32 ")
                    .s(r).s(", ").s(o).c(';');
                put(b);
                sv = r;
                sty = "u64";
            } else {
                sv = opnd(a);
                sty = ptx_type(at);
            }
            Str slot;
            if (i == 0) {
                slot = reg(vl);
            } else {
                uint32_t offv = new_value(nm2("_va_off_", n, "_", i), lptr);
                Str r = reg(offv);
                Str base = reg(vl);
                SB b = sb();
                b.s("    add.u64 ").s(r).s(", ").s(base).s(", ").i(8 * (pyint)i).c(';');
                put(b);
                slot = r;
            }
            SB b = sb();
            b.s("    st.local.").s(sty).s(" [").s(slot).s("], ").s(sv).c(';');
            put(b);
        }
        uint32_t vg = new_value(nm("_valist_gen_", n), vptr);
        Str r = reg(vg);
        Str lr = reg(vl);
        SB b = sb();
        b.s("    cvta.local.u64 ").s(r).s(", ").s(lr).c(';');
        put(b);
        va = r;
    } else {
        uint32_t nv = new_value(nm("_valist_null_", n), gptr);
        Str r = reg(nv);
        SB b = sb();
        b.s("    mov.u64 ").s(r).s(", 0;");
        put(b);
        va = r;
    }
    uint32_t rv = new_value(nm("_vprintf_rv_", n), S_INT32);
    put("    {");
    SB b0 = sb();
    b0.s("    .param .b64 _p0_").i(n).c(';');
    put(b0);
    SB b1 = sb();
    b1.s("    .param .b64 _p1_").i(n).c(';');
    put(b1);
    SB b2 = sb();
    b2.s("    .param .b32 _rv_").i(n).c(';');
    put(b2);
    Str far = reg(fa);
    SB b3 = sb();
    b3.s("    st.param.b64 [_p0_").i(n).s("], ").s(far).c(';');
    put(b3);
    SB b4 = sb();
    b4.s("    st.param.b64 [_p1_").i(n).s("], ").s(va).c(';');
    put(b4);
    SB b5 = sb();
    b5.s("    call.uni (_rv_").i(n).s("), vprintf, (_p0_").i(n).s(", _p1_").i(n).s(");");
    put(b5);
    Str rr = reg(rv);
    SB b6 = sb();
    b6.s("    ld.param.b32 ").s(rr).s(", [_rv_").i(n).s("];");
    put(b6);
    put("    }");
}

// Inline PTX (emit.py:1151-1168): %N -> the N-th operand (outputs, then
// inputs; replaced from the highest N down), then one line per
// ';'-separated statement, stripped of surrounding whitespace.
OCB_HD inline void Emit::emit_asm(const Inst &in) {
    uint32_t n = in.args.n;
    Str *ops = (Str *)tmp.alloc(sizeof(Str) * (n + 1), 8);
    if (!ops) { unsup(); return; }
    for (uint32_t q = 0; q < n; ++q) ops[q] = q < in.pidx ? reg(in.args[q]) : opnd(in.args[q]);
    for (uint32_t q = 0; q < in.func.n; ++q)
        if ((uint8_t)in.func.p[q] >= 0x80) { unsup(); return; }  // str.strip()'s Unicode set
    Str t = in.func;
    for (uint32_t q = n; q-- > 0;) {
        SB key = sb();
        key.c('%').i(q);
        Str kk = key.str();
        SB r = sb();
        bool any = false;
        for (uint32_t i = 0; i < t.n;) {
            if (i + kk.n <= t.n && mem_eq(t.p + i, kk.p, kk.n)) {
                r.s(ops[q]);
                i += kk.n;
                any = true;
            } else {
                r.c(t.p[i++]);
            }
        }
        if (any) t = r.str();
    }
    auto ws = [](char c) { return c == ' ' || (c >= 9 && c <= 13) || (c >= 0x1c && c <= 0x1f); };
    uint32_t st = 0;
    for (uint32_t i = 0; i <= t.n; ++i) {
        if (i < t.n && t.p[i] != ';') continue;
        uint32_t a = st, e = i;
        while (a < e && ws(t.p[a])) ++a;
        while (e > a && ws(t.p[e - 1])) --e;
        if (e > a) {
            SB b = sb();
            b.s("    ").s(Str{t.p + a, e - a}).c(';');
            put(b);
        }
        st = i + 1;
    }
}

// The label table of the kernel being emitted: open addressing over labels,
// filled on first use with every block label and branch target.
OCB_HD inline Emit::LblEnt *Emit::label_slot(Str l, bool create) {
    if (!lt_ok) {
        lt_ok = true;
        uint32_t want = 3 * k->blocks.n + 8;
        lt_cap = 16;
        while (lt_cap < 2 * want) lt_cap *= 2;
        lt = (LblEnt *)tmp.alloc(sizeof(LblEnt) * (uint64_t)lt_cap, 16);
        if (!lt) { lt_cap = 0; unsup(); return nullptr; }
        for (uint32_t i = 0; i < lt_cap; ++i) lt[i] = LblEnt{Str{nullptr, 0}, -1, 0};
        for (uint32_t i = 0; i < k->blocks.n; ++i) {  // the last block with a label wins
            LblEnt *e = label_slot(B(k->blocks[i]).label, true);
            if (e) e->blk = (int32_t)k->blocks[i];
        }
        for (uint32_t i = 0; i < k->blocks.n; ++i) {  // a CondBrTerm counts once per label
            const Term &t = B(k->blocks[i]).term;
            if (t.kind == T_BR) {
                LblEnt *e = label_slot(t.t, true);
                if (e) e->preds++;
            } else if (t.kind == T_CBR) {
                LblEnt *e = label_slot(t.t, true);
                if (e) e->preds++;
                if (!eq(t.f, t.t)) {
                    e = label_slot(t.f, true);
                    if (e) e->preds++;
                }
            }
        }
    }
    if (!lt_cap) return nullptr;
    uint32_t h = hash(l) & (lt_cap - 1);
    while (lt[h].l.p) {
        if (eq(lt[h].l, l)) return &lt[h];
        h = (h + 1) & (lt_cap - 1);
    }
    if (!create) return nullptr;
    lt[h].l = l;
    return &lt[h];
}
OCB_HD inline int32_t Emit::block_by_label(Str l) {
    LblEnt *e = label_slot(l, false);
    return e ? e->blk : -1;
}
// number of blocks whose terminator targets `l` (a CondBrTerm counts once)
OCB_HD inline uint32_t Emit::pred_count_of(Str l) {
    LblEnt *e = label_slot(l, false);
    return e ? e->preds : 0;
}

// ---- _emit_term (emit.py:2887-3123) --------------------------------------------
OCB_HD inline void Emit::emit_term(const Term &t) {
    if (t.kind == T_RET) {
        if (t.v.k != O_NONE) {
            Str val = opnd(t.v);
            const char *pt = ptx_type(m.opty(t.v));
            if (cstr_eq(pt, "f16")) pt = "b16";
            SB b = sb();
            b.s("    st.param.").s(pt).s(" [retval0], ").s(val).c(';');
            put(b);
        }
        put("    ret;");
        return;
    }
    if (t.kind == T_BR) {
        if (skip.has(t.t)) {
            int32_t tb = block_by_label(t.t);
            if (tb >= 0 && B((uint32_t)tb).term.kind == T_RET) {
                put("    ret;");
                return;
            }
        }
        SB b = sb();
        b.s("    bra ").s(t.t).c(';');
        put(b);
        return;
    }
    if (t.kind != T_CBR) {
        unsup();
        return;
    }
    if (t.v.k == O_VAL) {
        int32_t tb = block_by_label(t.t), fb = block_by_label(t.f);
        // edge counts of the two arms
        uint32_t ec_t = 0, ec_f = 0;
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            const Term &x = B(k->blocks[i]).term;
            if (x.kind == T_BR) {
                ec_t += eq(x.t, t.t);
                ec_f += eq(x.t, t.f);
            } else if (x.kind == T_CBR) {
                ec_t += eq(x.t, t.t) + eq(x.f, t.t);
                ec_f += eq(x.t, t.f) + eq(x.f, t.f);
            }
        }
        bool diamond = false;
        if (tb >= 0 && fb >= 0) {
            Block &T = B((uint32_t)tb), &F = B((uint32_t)fb);
            if (T.insts.n == 1 && F.insts.n == 1 && T.term.kind == T_BR && F.term.kind == T_BR &&
                eq(T.term.t, F.term.t) && I(T.insts[0]).kind == I_BIN && I(F.insts[0]).kind == I_BIN &&
                V((uint32_t)I(T.insts[0]).dest).id == V((uint32_t)I(F.insts[0]).dest).id && ec_t == 1 &&
                ec_f == 1)
                diamond = true;
        }
        if (diamond) {
            const Inst ti = I(B((uint32_t)tb).insts[0]), fi = I(B((uint32_t)fb).insts[0]);
            Str merge = B((uint32_t)tb).term.t;
            Str dest = reg(ti.dest);
            const char *pt = ptx_mov_type(V((uint32_t)ti.dest).ty);
            Str pred;
            if (is_pred(vid(t.v))) {
                pred = reg(t.v);
            } else {
                pred = fresh_pred();
                const char *ct = ptx_type(V(t.v.x).ty);
                Str src = reg(t.v);
                SB b = sb();
                b.s("    setp.ne.").s(ct).c(' ').s(pred).s(", ").s(src).s(", 0;");
                put(b);
            }
            Str top = opnd(ti.a);
            Str fop = opnd(fi.a);
            auto assign = [&](bool neg, Opnd src_lhs, Str sop) {
                SB g = sb();
                if (neg) g.c('!');
                g.s(pred);
                SB b = sb();
                if (src_lhs.k == O_VAL && is_pred(vid(src_lhs))) {
                    b.s("    @").s(g.str()).s(" selp.").s(pt).c(' ').s(dest).s(", 1, 0, ").s(sop).c(';');
                    put(b);
                    return;
                }
                if (src_lhs.k == O_VAL && !is_ptr(V(src_lhs.x).ty)) {
                    const char *sp = ptx_type(V(src_lhs.x).ty);
                    const char *ints = " s8 u8 s16 u16 s32 u32 s64 u64 ";
                    if (cstr_in(sp, ints) && cstr_in(pt, ints) && !cstr_eq(sp, pt)) {
                        b.s("    @").s(g.str()).s(" cvt.").s(pt).c('.').s(sp).c(' ').s(dest).s(", ").s(sop).c(';');
                        put(b);
                        return;
                    }
                }
                b.s("    @").s(g.str()).s(" mov.").s(pt).c(' ').s(dest).s(", ").s(sop).c(';');
                put(b);
            };
            assign(false, ti.a, top);
            assign(true, fi.a, fop);
            skip.add(t.t);
            skip.add(t.f);
            int32_t mb = block_by_label(merge);
            uint32_t mpc = mb >= 0 ? pred_count_of(merge) : 0;
            if (mb >= 0 && mpc == 2) {
                skip.add(merge);
                Block &M = B((uint32_t)mb);
                for (uint32_t q = 0; q < M.insts.n && !bad(); ++q) emit_inst(M.insts[q]);
                if (M.term.kind != T_NONE) {
                    if (++term_depth > 24) { unsup(); return; }
                    emit_term(M.term);
                    --term_depth;
                }
            } else {
                SB b = sb();
                b.s("    bra ").s(merge).c(';');
                put(b);
            }
            return;
        }
        Str pred;
        if (is_pred(vid(t.v))) {
            pred = reg(t.v);
        } else {
            pred = fresh_pred();
            const char *ct = ptx_type(V(t.v.x).ty);
            Str src = reg(t.v);
            SB b = sb();
            b.s("    setp.ne.").s(ct).c(' ').s(pred).s(", ").s(src).s(", 0;");
            put(b);
        }
        bool false_is_ret = fb >= 0 && B((uint32_t)fb).insts.n == 0 && B((uint32_t)fb).term.kind == T_RET;
        if (false_is_ret) {
            uint32_t tpc = pred_count_of(t.t);
            bool self_loop = false;
            if (tb >= 0) {
                const Term &x = B((uint32_t)tb).term;
                self_loop = (x.kind == T_BR && eq(x.t, t.t)) ||
                            (x.kind == T_CBR && (eq(x.t, t.t) || eq(x.f, t.t)));
            }
            if (tpc == 1 && !self_loop) {
                SB b = sb();
                b.s("    @!").s(pred).s(" ret;");
                put(b);
                if (pred_count_of(t.f) <= 1) skip.add(t.f);
                skip.add(t.t);
                if (tb >= 0) {
                    Block &T = B((uint32_t)tb);
                    for (uint32_t q = 0; q < T.insts.n && !bad(); ++q) emit_inst(T.insts[q]);
                    if (T.term.kind == T_BR) {
                        Str ml = T.term.t;
                        int32_t mb = block_by_label(ml);
                        uint32_t mpc = pred_count_of(ml);
                        if (mb >= 0 && B((uint32_t)mb).insts.n == 0 && B((uint32_t)mb).term.kind == T_RET &&
                            mpc == 1) {
                            skip.add(ml);
                            put("    ret;");
                        } else {
                            if (++term_depth > 24) { unsup(); return; }
                            emit_term(T.term);
                            --term_depth;
                        }
                    } else if (T.term.kind != T_NONE) {
                        if (++term_depth > 24) { unsup(); return; }
                        emit_term(T.term);
                        --term_depth;
                    }
                }
                return;
            }
            SB b = sb();
            b.s("    @").s(pred).s(" bra ").s(t.t).c(';');
            put(b);
            SB b2 = sb();
            b2.s("    bra ").s(t.f).c(';');
            put(b2);
            return;
        }
        SB b = sb();
        b.s("    @").s(pred).s(" bra ").s(t.t).c(';');
        put(b);
        SB b2 = sb();
        b2.s("    bra ").s(t.f).c(';');
        put(b2);
        return;
    }
    if (t.v.k == O_CONST && !pv_eq_int(pv_of(m.consts[t.v.x]), 0)) {
        SB b = sb();
        b.s("    bra ").s(t.t).c(';');
        put(b);
    } else {
        SB b = sb();
        b.s("    bra ").s(t.f).c(';');
        put(b);
    }
}

OCB_HD inline void Emit::emit_block(uint32_t bidx) {
    Block &b = B(bidx);
    if (skip.has(b.label)) return;
    bool is_entry = eq(b.label, "entry") || sstarts(b.label, "entry_");
    if (!is_entry) {
        SB s = sb();
        s.s(b.label).c(':');
        put(s);
    }
    for (uint32_t q = 0; q < b.insts.n && !bad(); ++q) emit_inst(b.insts[q]);
    if (b.term.kind != T_NONE && !bad()) emit_term(b.term);
}

}  // namespace cc
}  // namespace ocb
