// Parser, expressions: parser.py:368-2249 restated for the supported subset.
#pragma once
#include "cc_parse.cuh"

namespace ocb {
namespace cc {

// str.isupper() for an identifier token of <= 2 chars (template parameter
// heuristic of _parse_type, parser.py:464-468)
OCB_HD inline bool py_isupper(Str s) {
    bool cased = false;
    for (uint32_t i = 0; i < s.n; ++i) {
        char c = s.p[i];
        if (c >= 'a' && c <= 'z') return false;
        if (c >= 'A' && c <= 'Z') cased = true;
    }
    return cased;
}

// typedef names registered in Parser.__init__ (parser.py:73-86)
OCB_HD inline bool typedef_scalar(Str v, Ty &t) {
    if (eq(v, "bool")) { t = S_INT32; return true; }
    if (eq(v, "size_t") || eq(v, "uintptr_t") || eq(v, "uint64_t")) { t = S_UINT64; return true; }
    if (eq(v, "ptrdiff_t") || eq(v, "intptr_t") || eq(v, "int64_t")) { t = S_INT64; return true; }
    if (eq(v, "int8_t") || eq(v, "int16_t") || eq(v, "int32_t")) { t = S_INT32; return true; }
    if (eq(v, "uint8_t") || eq(v, "uint16_t") || eq(v, "uint32_t")) { t = S_UINT32; return true; }
    return false;
}


// _parse_type (parser.py:368-472)
OCB_HD inline bool Parser::parse_type(Ty &out) {
    while (peek() == TK_VOLATILE || peek() == TK_CONST) advance();
    uint32_t k = peek();
    switch (k) {
    case TK_VOID: advance(); out = S_VOID; return true;
    case TK_FLOAT: advance(); out = S_FLOAT; return true;
    case TK_DOUBLE: advance(); out = S_DOUBLE; return true;
    case TK_HALF: advance(); out = S_HALF; return true;
    case TK_INT: advance(); out = S_INT32; return true;
    case TK_UNSIGNED:
        advance();
        if (match(TK_INT)) {
        } else if (match(TK_SHORT)) {
            match(TK_INT);
            out = S_UINT16;
            return true;
        } else if (match(TK_CHAR)) {
            out = S_UINT8;
            return true;
        } else if (match(TK_LONG)) {
            if (match(TK_LONG)) {
                match(TK_INT);
                out = S_UINT64;
                return true;
            }
            match(TK_INT);
        }
        out = S_UINT32;
        return true;
    case TK_LONG:
        advance();
        if (match(TK_LONG)) {
            match(TK_INT);
            out = S_INT64;
            return true;
        }
        match(TK_INT);
        out = S_INT32;
        return true;
    case TK_SHORT: advance(); match(TK_INT); out = S_INT16; return true;
    case TK_SIGNED:
        advance();
        if (match(TK_CHAR)) { out = S_INT8; return true; }
        if (match(TK_SHORT)) { match(TK_INT); out = S_INT16; return true; }
        if (match(TK_LONG)) {
            if (match(TK_LONG)) { match(TK_INT); out = S_INT64; return true; }
            match(TK_INT);
            out = S_INT32;
            return true;
        }
        match(TK_INT);
        out = S_INT32;
        return true;
    case TK_CHAR: advance(); out = S_INT8; return true;
    case TK_BOOL: advance(); out = S_INT32; return true;
    default: break;
    }
    if (k == TK_STRUCT || k == TK_UNION) {  // a defined struct or union
        advance();
        if (!at(TK_IDENT)) {
            perr();
            return false;
        }
        Str sn = peekv();
        advance();
        if (find_struct(sn, out)) return true;
        perr();
        return false;
    }
    if (k == TK_ENUM) {
        advance();
        if (at(TK_IDENT)) advance();
        out = S_INT32;
        return true;
    }
    if (k == TK_IDENT) {
        Str v = peekv();
        Ty t;
        if (user_typedef(v, t) || typedef_scalar(v, t) || vector_type(v, t) ||
            user_struct(v, t)) {  // _typedefs, then a bare struct name
            advance();
            out = t;
            return true;
        }
        if (v.n <= 2 && py_isupper(v)) {
            advance();
            out = S_FLOAT;
            return true;
        }
    }
    perr();
    return false;
}

// _parse_type_with_ptr (parser.py:474-508)
OCB_HD inline bool Parser::parse_type_with_ptr(Ty &out) {
    match(TK_STATIC);
    bool pv = match(TK_VOLATILE);
    bool pc = match(TK_CONST);
    if (match(TK_VOLATILE)) pv = true;
    match(TK_STATIC);
    Ty base;
    if (!parse_type(base)) return false;
    if (match(TK_CONST)) pc = true;
    if (match(TK_VOLATILE)) pv = true;
    while (match(TK_STAR)) {
        match(TK_CONST);
        match(TK_VOLATILE);
        bool ok = true;
        base = ty_ptr(base, AS_GLOBAL, pv, ok);
        if (!ok) { unsup(); return false; }
        pv = false;
    }
    bool restrict_ = at(TK_IDENT) && eq(peekv(), "__restrict__");
    if (restrict_) advance();
    if (pc && restrict_ && is_ptr(base)) base = (base & ~(7u << 6)) | (AS_CONST << 6);
    out = base;
    return true;
}

OCB_HD inline Opnd Parser::parse_expr() {
    Opnd r = parse_assign_expr();
    while (!bad() && match(TK_COMMA)) r = parse_assign_expr();
    return r;
}

// _parse_assign_expr (parser.py:521-692)
OCB_HD inline Opnd Parser::parse_assign_expr() {
    if (++nest > MAX_NEST) { unsup(); --nest; return onone(); }
    Str lhs_orig{nullptr, 0};
    if (at(TK_IDENT)) {
        Str cand = peekv();
        uint32_t np = pos + 1;
        if (np < tk.n && is_assign_op(kind_at(np)) && vars.has(cand)) {
            lhs_orig = cand;
        } else if (np < tk.n && kind_at(np) == TK_DOT && vars.has(cand) &&
                   isstruct(*vars.get(cand))) {
            // struct.field = val: the per-field variable is the target
            uint32_t fp = np + 1;
            if (fp < tk.n && kind_at(fp) == TK_IDENT && fp + 1 < tk.n &&
                is_assign_op(kind_at(fp + 1))) {
                Str cn = cat(ar, cand, S("_"), val_at(fp));
                if (vars.has(cn)) lhs_orig = cn;
            }
        }
    }
    Opnd lhs = parse_or_expr();
    Opnd result = lhs;
    if (bad()) goto out;
    if (match(TK_QUESTION)) {
        Opnd tv = parse_expr();
        if (bad() || !expect(TK_COLON)) goto out;
        Opnd fv = parse_assign_expr();
        if (bad()) goto out;
        Ty rt = result_type(tv, fv);
        uint32_t dest = new_val("ternary", rt);
        if (bad()) goto out;  // outside a kernel: AttributeError in new_value
        uint32_t tb = new_block("tern_true"), fb = new_block("tern_false"),
                 mb = new_block("tern_merge");
        B().term = Term{T_CBR, lhs, m.blocks[tb].label, m.blocks[fb].label};
        cur = tb;
        emit_bin(dest, BO_ADD, tv, m.czero(rt));
        m.blocks[tb].term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
        cur = fb;
        emit_bin(dest, BO_ADD, fv, m.czero(rt));
        m.blocks[fb].term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
        cur = mb;
        result = ov(dest);
        goto out;
    }
    if (match(TK_ASSIGN)) {
        Opnd rhs = parse_assign_expr();
        if (bad()) goto out;
        if (isval(lhs) && is_ptr(tyof(lhs))) {
            if (lhs_orig.p && vars.has(lhs_orig) && !shared_scalars.has(lhs_orig)) {
                vars.set(ar, lhs_orig, rhs);
                result = rhs;
                goto out;
            }
            Ty pt = ty_pointee(tyof(lhs));
            Ty rt = tyof(rhs);
            if (isval(rhs) && is_scalar_ty(rt) && is_scalar_ty(pt) && rt != pt) {
                uint32_t co = new_val("coerce", pt);
                emit_cvt(co, rhs);
                rhs = ov(co);
            } else if (iscon(rhs) && is_scalar_ty(pt) && !is_ptr(rt) && rt != pt && !ty_is_float(rt) &&
                       !ty_is_float(pt)) {
                Const c = m.consts[rhs.x];
                c.ty = pt;
                m.consts.push(ar, c);
                rhs = oc(m.consts.n - 1);
            }
            emit_store(lhs, rhs);
            result = rhs;
            goto out;
        }
        Str un = lhs_orig.p ? lhs_orig : (isval(lhs) ? vname(lhs) : Str{nullptr, 0});
        if (un.p && vars.has(un)) {
            Opnd prev = *vars.get(un);
            if (prev.k == O_VAL && is_scalar_ty(tyof(prev)) && (rhs.k == O_VAL || rhs.k == O_CONST) &&
                is_scalar_ty(tyof(rhs))) {
                if (iscon(rhs) || (isval(rhs) && !eq(vname(rhs), un))) {
                    Ty pt = tyof(prev);
                    uint32_t mat = new_val(un, pt);
                    emit_bin(mat, BO_ADD, rhs, m.czero(pt));
                    rhs = ov(mat);
                }
            }
            vars.set(ar, un, rhs);
            if (isstruct(rhs)) copy_struct_fields(rhs.x, un);
        }
        result = rhs;
        goto out;
    }
    {
        static const uint32_t toks[] = {TK_PLUS_EQ, TK_MINUS_EQ, TK_STAR_EQ, TK_SLASH_EQ,
                                        TK_PERCENT_EQ, TK_AMP_EQ, TK_PIPE_EQ, TK_CARET_EQ,
                                        TK_LSHIFT_EQ, TK_RSHIFT_EQ};
        static const uint8_t ops[] = {BO_ADD, BO_SUB, BO_MUL, BO_DIV, BO_MOD,
                                      BO_AND, BO_OR, BO_XOR, BO_SHL, BO_SHR};
        for (int k = 0; k < 10; ++k) {
            if (match(toks[k])) {
                Opnd rhs = parse_assign_expr();
                if (bad()) goto out;
                if (isval(lhs)) {
                    uint32_t nv = new_val(cat(ar, vname(lhs), S("_compound")), tyof(lhs));
                    emit_bin(nv, ops[k], lhs, rhs);
                    Str un = lhs_orig.p ? lhs_orig : vname(lhs);
                    if (vars.has(un)) vars.set(ar, un, ov(nv));
                    result = ov(nv);
                    goto out;
                }
            }
        }
    }
out:
    --nest;
    return result;
}

// _parse_or_expr / _parse_and_expr (parser.py:694-782): short-circuit blocks
OCB_HD inline Opnd Parser::parse_or_expr() {
    Opnd lhs = parse_and_expr();
    while (!bad() && match(TK_OR)) {
        uint32_t dest = new_val("lor", S_INT32);
        if (bad()) return lhs;  // outside a kernel: AttributeError in new_value
        uint32_t rb = new_block("lor_rhs"), sb = new_block("lor_skip"), mb = new_block("lor_merge");
        B().term = Term{T_CBR, lhs, m.blocks[sb].label, m.blocks[rb].label};
        VarMap before = vars.copy(ar);
        cur = rb;
        Opnd rhs = parse_and_expr();
        if (bad()) return lhs;
        emit_bin(dest, BO_ADD, rhs, m.cint(S_INT32, 0));
        B().term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
        struct RB { Opnd nv, old; };
        Vec<RB> reb;
        reb.init();
        for (uint32_t i = 0; i < vars.e.n; ++i) {
            const VarEnt &en = vars.e[i];
            if (!en.live || en.v.k != O_VAL) continue;
            Opnd *o = before.get(en.name);
            if (!o || o->k != O_VAL || o->x == en.v.x) continue;
            reb.push(ar, RB{en.v, *o});
        }
        cur = sb;
        emit_bin(dest, BO_ADD, m.cint(S_INT32, 1), m.cint(S_INT32, 0));
        for (uint32_t i = 0; i < reb.n; ++i)
            emit_bin(reb[i].nv.x, BO_ADD, reb[i].old, m.czero(tyof(reb[i].nv)));
        B().term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
        cur = mb;
        lhs = ov(dest);
    }
    return lhs;
}

OCB_HD inline Opnd Parser::parse_and_expr() {
    Opnd lhs = parse_bitor_expr();
    while (!bad() && match(TK_AND)) {
        uint32_t dest = new_val("land", S_INT32);
        if (bad()) return lhs;  // outside a kernel: AttributeError in new_value
        uint32_t rb = new_block("land_rhs"), sb = new_block("land_skip"), mb = new_block("land_merge");
        B().term = Term{T_CBR, lhs, m.blocks[rb].label, m.blocks[sb].label};
        VarMap before = vars.copy(ar);
        cur = rb;
        Opnd rhs = parse_bitor_expr();
        if (bad()) return lhs;
        emit_bin(dest, BO_ADD, rhs, m.cint(S_INT32, 0));
        B().term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
        struct RB { Opnd nv, old; };
        Vec<RB> reb;
        reb.init();
        for (uint32_t i = 0; i < vars.e.n; ++i) {
            const VarEnt &en = vars.e[i];
            if (!en.live || en.v.k != O_VAL) continue;
            Opnd *o = before.get(en.name);
            if (!o || o->k != O_VAL || o->x == en.v.x) continue;
            reb.push(ar, RB{en.v, *o});
        }
        cur = sb;
        emit_bin(dest, BO_ADD, m.cint(S_INT32, 0), m.cint(S_INT32, 0));
        for (uint32_t i = 0; i < reb.n; ++i)
            emit_bin(reb[i].nv.x, BO_ADD, reb[i].old, m.czero(tyof(reb[i].nv)));
        B().term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
        cur = mb;
        lhs = ov(dest);
    }
    return lhs;
}

#define OCB_BITLEVEL(FN, NEXT, TOK, OP, NAME)                          \
    OCB_HD inline Opnd Parser::FN() {                                  \
        Opnd lhs = NEXT();                                             \
        while (!bad() && match(TOK)) {                                 \
            Opnd rhs = NEXT();                                         \
            if (bad()) return lhs;                                     \
            Opnd f;                                                    \
            if (const_fold(OP, lhs, rhs, f)) {                         \
                lhs = f;                                               \
            } else {                                                   \
                uint32_t d = new_val(NAME, result_type(lhs, rhs));    \
                emit_bin(d, OP, lhs, rhs);                             \
                lhs = ov(d);                                           \
            }                                                          \
        }                                                              \
        return lhs;                                                    \
    }
OCB_BITLEVEL(parse_bitor_expr, parse_bitxor_expr, TK_PIPE, BO_OR, "bitor")
OCB_BITLEVEL(parse_bitxor_expr, parse_bitand_expr, TK_CARET, BO_XOR, "bitxor")
OCB_BITLEVEL(parse_bitand_expr, parse_cmp_expr, TK_AMP, BO_AND, "bitand")
#undef OCB_BITLEVEL

// _parse_cmp_expr (parser.py:823-839): one comparison, its RHS an add-expr
OCB_HD inline Opnd Parser::parse_cmp_expr() {
    Opnd lhs = parse_shift_expr();
    if (bad()) return lhs;
    static const uint32_t toks[] = {TK_EQ, TK_NE, TK_LT, TK_LE, TK_GT, TK_GE};
    static const uint8_t ops[] = {CO_EQ, CO_NE, CO_LT, CO_LE, CO_GT, CO_GE};
    for (int k = 0; k < 6; ++k) {
        if (match(toks[k])) {
            Opnd rhs = parse_add_expr();
            if (bad()) return lhs;
            uint32_t d = new_val("cmp", S_BOOL);
            emit_cmp(d, ops[k], lhs, rhs);
            return ov(d);
        }
    }
    return lhs;
}

OCB_HD inline Opnd Parser::parse_shift_expr() {
    Opnd lhs = parse_add_expr();
    for (;;) {
        if (bad()) return lhs;
        uint8_t op;
        const char *nm;
        if (match(TK_LSHIFT)) { op = BO_SHL; nm = "shl"; }
        else if (match(TK_RSHIFT)) { op = BO_SHR; nm = "shr"; }
        else break;
        Opnd rhs = parse_add_expr();
        if (bad()) return lhs;
        Opnd f;
        if (const_fold(op, lhs, rhs, f)) {
            lhs = f;
        } else {
            Ty lt = (isval(lhs) || iscon(lhs)) ? tyof(lhs) : (Ty)S_INT32;
            uint32_t d = new_val(nm, lt);
            emit_bin(d, op, lhs, rhs);
            lhs = ov(d);
        }
    }
    return lhs;
}

OCB_HD inline Opnd Parser::parse_add_expr() {
    Opnd lhs = parse_mul_expr();
    for (;;) {
        if (bad()) return lhs;
        if (match(TK_PLUS)) {
            Opnd rhs = parse_mul_expr();
            if (bad()) return lhs;
            Ty lt = tyof(lhs), rt = tyof(rhs);
            if (is_ptr(lt) && !is_ptr(rt)) rhs = scale_ptr_off(lt, rhs);
            else if (is_ptr(rt) && !is_ptr(lt)) lhs = scale_ptr_off(rt, lhs);
            Opnd f;
            if (const_fold(BO_ADD, lhs, rhs, f)) {
                lhs = f;
            } else {
                uint32_t d = new_val("add", result_type(lhs, rhs));
                emit_bin(d, BO_ADD, lhs, rhs);
                lhs = ov(d);
            }
        } else if (match(TK_MINUS)) {
            Opnd rhs = parse_mul_expr();
            if (bad()) return lhs;
            Ty lt = tyof(lhs), rt = tyof(rhs);
            if (is_ptr(lt) && !is_ptr(rt)) rhs = scale_ptr_off(lt, rhs);
            Opnd f;
            if (const_fold(BO_SUB, lhs, rhs, f)) {
                lhs = f;
            } else {
                uint32_t d = new_val("sub", result_type(lhs, rhs));
                emit_bin(d, BO_SUB, lhs, rhs);
                lhs = ov(d);
            }
        } else {
            break;
        }
    }
    return lhs;
}

OCB_HD inline Opnd Parser::parse_mul_expr() {
    Opnd lhs = parse_unary_expr();
    for (;;) {
        if (bad()) return lhs;
        uint8_t op;
        const char *nm;
        if (match(TK_STAR)) { op = BO_MUL; nm = "mul"; }
        else if (match(TK_SLASH)) { op = BO_DIV; nm = "div"; }
        else if (match(TK_PERCENT)) { op = BO_MOD; nm = "mod"; }
        else break;
        Opnd rhs = parse_unary_expr();
        if (bad()) return lhs;
        Opnd f;
        if (const_fold(op, lhs, rhs, f)) {
            lhs = f;
        } else {
            uint32_t d = new_val(nm, result_type(lhs, rhs));
            emit_bin(d, op, lhs, rhs);
            lhs = ov(d);
        }
    }
    return lhs;
}

// &x of a scalar (parser.py:1054-1069, 1156-1170): the slot `_spill_<x>` is
// a .local declaration of one element, made on first use and kept in the
// variable table; each `&` stores the current value into it.  Later reads of
// x do not see writes through the pointer, except after an inlined call that
// received it (inline_call reloads those).
OCB_HD inline Opnd Parser::spill_scalar(Str name, Opnd value) {
    Str sn = cat(ar, S("_spill_"), name);
    Opnd *sp = vars.get(sn);
    Opnd slot;
    if (sp) {
        slot = *sp;
    } else {
        Ty vt = tyof(value);
        bool ok = true;
        Ty lt = ty_ptr(vt, AS_LOCAL, false, ok);
        if (!ok) {
            unsup();
            return onone();
        }
        uint32_t v = new_val(sn, lt);
        slot = ov(v);
        vars.set(ar, sn, slot);
        kern->locals.push(ar, LocalDecl{sn, vt, 1, v});
    }
    emit_store(slot, value);
    return slot;
}

// _parse_unary_expr (parser.py:972-1287)
OCB_HD inline Opnd Parser::parse_unary_expr() {
    if (++nest > MAX_NEST) { unsup(); --nest; return onone(); }
    Opnd r = onone();
    if (match(TK_AMP)) {
        bool generic = true;
        if (at(TK_IDENT)) {
            Str name = peekv();
            Opnd *gs = global_consts.get(name);
            if (gs && gs->k == O_SYM) {  // &global, &global[idx] (parser.py:978-1016)
                uint32_t gi = gs->x;
                advance();
                Opnd addr = gaddr(gi);
                if (match(TK_LBRACKET)) {
                    Opnd index = parse_expr();
                    if (bad() || !expect(TK_RBRACKET)) { --nest; return onone(); }
                    Ty gp = m.gvars[gi].ptr;
                    uint32_t es = m.tsize(ty_pointee(gp));
                    if (es != 1) {
                        Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                        uint32_t sc = new_val("scale", it);
                        emit_bin(sc, BO_MUL, index, m.cint(it, es));
                        index = ov(sc);
                    }
                    uint32_t ea = new_val("elem_addr", gp);
                    emit_bin(ea, BO_ADD, addr, index);
                    addr = field_chain(ov(ea), ty_pointee(gp), ty_as(gp));  // &g[i].f
                }
                --nest;
                return addr;
            }
            Opnd *vp = vars.get(name);
            if (vp) {
                Opnd var = *vp;
                Ty vt = tyof(var);
                if (is_ptr(vt)) {
                    advance();
                    if (match(TK_LBRACKET)) {
                        Opnd index = parse_expr();
                        if (bad() || !expect(TK_RBRACKET)) goto out;
                        uint32_t es = m.tsize(ty_pointee(vt));
                        if (es != 1) {
                            Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                            uint32_t s = new_val("scale", it);
                            emit_bin(s, BO_MUL, index, m.cint(it, es));
                            index = ov(s);
                        }
                        uint32_t a = new_val("addr", vt);
                        emit_bin(a, BO_ADD, var, index);
                        r = field_chain(ov(a), ty_pointee(vt), ty_as(vt));  // &a[i].f.g
                        goto out;
                    }
                    if (at(TK_ARROW) || at(TK_DOT)) {
                        pos -= 1;  // fall through to the generic handler
                    } else {
                        r = var;
                        goto out;
                    }
                } else if (ty_is_struct(vt)) {  // &s / &s.f[i] (parser.py:1074-1151)
                    uint32_t nk = pos + 1 < tk.n ? kind_at(pos + 1) : TK_EOF;
                    bool member = nk == TK_DOT || nk == TK_ARROW;
                    if (nk == TK_DOT && pos + 3 < tk.n && kind_at(pos + 2) == TK_IDENT &&
                        kind_at(pos + 3) == TK_LBRACKET) {
                        Opnd *fl = vars.get(cat(ar, name, S("_"), val_at(pos + 2)));
                        if (fl && fl->k == O_VAL && is_ptr(tyof(*fl))) {
                            Opnd flat = *fl;
                            pos += 4;
                            Opnd index = parse_expr();
                            if (bad() || !expect(TK_RBRACKET)) goto out;
                            uint32_t es = m.tsize(ty_pointee(tyof(flat)));
                            if (es != 1) {
                                Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                                uint32_t sc = new_val("scale", it);
                                emit_bin(sc, BO_MUL, index, m.cint(it, es));
                                index = ov(sc);
                            }
                            uint32_t a = new_val("addr", tyof(flat));
                            emit_bin(a, BO_ADD, flat, index);
                            r = ov(a);
                            goto out;
                        }
                    }
                    if (!member) {  // the struct spilled field by field to a .local slot
                        advance();
                        Str sn = cat(ar, S("_spill_"), name);
                        Opnd *sp = vars.get(sn);
                        Opnd slot;
                        if (sp) {
                            slot = *sp;
                        } else {
                            bool ok = true;
                            Ty lt = ty_ptr(vt, AS_LOCAL, false, ok);
                            if (!ok) { unsup(); goto out; }
                            uint32_t v = new_val(sn, lt);
                            slot = ov(v);
                            vars.set(ar, sn, slot);
                            kern->locals.push(ar, LocalDecl{sn, vt, 1, v});
                        }
                        uint32_t nf = m.nfields(vt);
                        for (uint32_t q = 0; q < nf && !bad(); ++q) {
                            SField fd = m.field(vt, q);
                            if (ty_is_struct(fd.ty)) continue;
                            Opnd *fv = vars.get(cat(ar, name, S("_"), fd.name));
                            if (!fv) continue;
                            Opnd fval = *fv;
                            bool ok = true;
                            Ty fp = ty_ptr(fd.ty, AS_LOCAL, false, ok);
                            if (!ok) { unsup(); goto out; }
                            uint32_t fa = new_val("faddr", fp);
                            emit_bin(fa, BO_ADD, slot, m.cint(S_INT32, m.field_offset(vt, q)));
                            emit_store(ov(fa), fval);
                        }
                        r = slot;
                        goto out;
                    }
                } else {  // &scalar: spilled to a one-element .local slot
                    advance();
                    r = spill_scalar(name, var);
                    goto out;
                }
            }
        }
        if (generic) {
            Opnd o = parse_unary_expr();
            if (bad()) goto out;
            if (o.k == O_VAL && is_ptr(tyof(o))) { r = o; goto out; }
            if (o.k == O_VAL && is_scalar_ty(tyof(o)) && kern) {  // &expr of a scalar: spilled too
                r = spill_scalar(vname(o), o);
                goto out;
            }
            r = o;
            goto out;
        }
    }
    if (match(TK_STAR)) {
        Opnd o = parse_unary_expr();
        if (bad()) goto out;
        if (o.k == O_VAL && is_ptr(tyof(o))) {
            uint32_t d = new_val("deref", ty_pointee(tyof(o)));
            emit_load(d, o);
            r = ov(d);
            goto out;
        }
        // not a pointer: the reference carries on with the next checks
    }
    if (match(TK_SIZEOF)) {
        // sizeof(type) or sizeof(expr); any exception in the type tries the expr
        if (!expect(TK_LPAREN)) goto out;
        uint32_t saved = pos;
        Ty st;
        int64_t size;
        if (parse_type_with_ptr(st)) {
            size = m.tsize(st);
        } else {
            if (!catch_any()) goto out;
            pos = saved;
            Opnd e = parse_expr();
            if (bad()) goto out;
            size = m.tsize((isval(e) || iscon(e)) ? tyof(e) : (Ty)S_INT32);
        }
        if (!expect(TK_RPAREN)) goto out;
        r = m.cint(S_INT32, size);
        goto out;
    }
    if (match(TK_PLUS)) { r = parse_unary_expr(); goto out; }
    if (match(TK_MINUS)) {
        Opnd o = parse_unary_expr();
        if (bad()) goto out;
        Ty t = (isval(o) || iscon(o)) ? tyof(o) : (Ty)S_INT32;
        Opnd zero = ty_is_float(t) ? m.cfloat(S_FLOAT, 0.0) : m.cint(t, 0);
        Opnd f;
        if (const_fold(BO_SUB, zero, o, f)) { r = f; goto out; }
        if (bad()) goto out;
        uint32_t d = new_val("neg", t);
        emit_bin(d, BO_SUB, zero, o);
        r = ov(d);
        goto out;
    }
    if (match(TK_TILDE)) {
        Opnd o = parse_unary_expr();
        if (bad()) goto out;
        Ty t = (isval(o) || iscon(o)) ? tyof(o) : (Ty)S_INT32;
        Opnd ones = !is_ptr(t) ? m.cint(t, -1) : m.cint(S_INT32, -1);
        Opnd f;
        if (const_fold(BO_XOR, o, ones, f)) { r = f; goto out; }
        if (bad()) goto out;
        uint32_t d = new_val("bnot", t);
        emit_bin(d, BO_XOR, o, ones);
        r = ov(d);
        goto out;
    }
    if (match(TK_BANG)) {
        Opnd o = parse_unary_expr();
        if (bad()) goto out;
        uint32_t d = new_val("lnot", S_BOOL);
        emit_cmp(d, CO_EQ, o, m.cint(S_INT32, 0));
        r = ov(d);
        goto out;
    }
    if (at(TK_PLUSPLUS) || at(TK_MINUSMINUS)) {
        bool inc = match(TK_PLUSPLUS);
        if (!inc) advance();
        Str pre{nullptr, 0};
        if (at(TK_IDENT)) pre = peekv();
        Opnd o = parse_unary_expr();
        if (bad()) goto out;
        if (o.k == O_VAL) {
            Ty t = tyof(o);
            Opnd step = is_ptr(t) ? scale_ptr_off(t, m.cint(S_INT32, 1)) : m.cint(t, 1);
            uint32_t nv = new_val(cat(ar, vname(o), S(inc ? "_preinc" : "_predec")), t);
            emit_bin(nv, inc ? BO_ADD : BO_SUB, o, step);
            Str un = vname(o);
            if (pre.p) {
                Opnd *pv = vars.get(pre);
                if (pv && pv->k == O_VAL && pv->x == o.x) un = pre;
            }
            vars.set(ar, un, ov(nv));
            r = ov(nv);
            goto out;
        }
        r = o;
        goto out;
    }
    if (at(TK_LPAREN)) {
        // cast: (type)expr; a ParseError anywhere inside restores the position
        uint32_t saved = pos;
        advance();
        Ty ct;
        bool ok = parse_type(ct);
        while (ok && match(TK_STAR)) {
            bool pok = true;
            ct = ty_ptr(ct, AS_GLOBAL, false, pok);
            if (!pok) { unsup(); goto out; }
        }
        if (ok && expect(TK_RPAREN)) {
            Opnd o = parse_unary_expr();
            if (!bad() && ty_is_struct(ct)) { unsup(); goto out; }  // CvtInst to a struct
            if (!bad()) {
                if (is_ptr(ct) && o.k == O_VAL && is_ptr(tyof(o)) && ty_as(tyof(o)) != AS_GLOBAL) {
                    bool pok = true;
                    ct = ty_ptr(ty_pointee(ct), ty_as(tyof(o)), false, pok);
                    if (!pok) { unsup(); goto out; }
                }
                uint32_t d = new_val("cast", ct);
                emit_cvt(d, o);
                r = ov(d);
                goto out;
            }
        }
        if (!catch_parse()) goto out;  // except ParseError: self._pos = saved
        pos = saved;
    }
    r = parse_postfix_expr();
out:
    --nest;
    return r;
}

// _parse_postfix_expr (parser.py:1289-1530)
OCB_HD inline Opnd Parser::parse_postfix_expr() {
    Str src_name{nullptr, 0};
    if (at(TK_IDENT) && vars.has(peekv())) src_name = peekv();
    Opnd lhs = parse_primary_expr();
    for (;;) {
        if (bad()) return lhs;
        if (at(TK_PLUSPLUS) || at(TK_MINUSMINUS)) {
            bool inc = at(TK_PLUSPLUS);
            advance();
            if (lhs.k == O_VAL) {
                Ty t = tyof(lhs);
                Opnd step = is_ptr(t) ? scale_ptr_off(t, m.cint(S_INT32, 1)) : m.cint(t, 1);
                uint32_t nv = new_val(cat(ar, vname(lhs), S(inc ? "_inc" : "_dec")), t);
                emit_bin(nv, inc ? BO_ADD : BO_SUB, lhs, step);
                Str un = src_name.p ? src_name : vname(lhs);
                vars.set(ar, un, ov(nv));
            }
            src_name = Str{nullptr, 0};
            continue;
        }
        if (match(TK_LBRACKET)) {
            Opnd index = parse_expr();
            if (bad() || !expect(TK_RBRACKET)) return lhs;
            if (lhs.k == O_VAL && is_ptr(tyof(lhs))) {
                Ty lt = tyof(lhs);
                Opnd *rs = row_strides.get(vname(lhs));
                if (rs && at(TK_LBRACKET)) {
                    Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                    uint32_t s = new_val("scale", it);
                    emit_bin(s, BO_MUL, index, m.cint(it, m.consts[rs->x].i));
                    uint32_t a = new_val("addr", lt);
                    emit_bin(a, BO_ADD, lhs, ov(s));
                    lhs = ov(a);
                    continue;
                }
                Ty pt = ty_pointee(lt);
                uint32_t es = m.tsize(pt);
                if (es != 1) {
                    Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                    uint32_t s = new_val("scale", it);
                    emit_bin(s, BO_MUL, index, m.cint(it, es));
                    index = ov(s);
                }
                uint32_t a = new_val("addr", lt);
                emit_bin(a, BO_ADD, lhs, index);
                if (ty_is_struct(pt) || is_assign_op(peek())) {  // struct element: an address
                    lhs = ov(a);
                } else {
                    uint32_t d = new_val("elem", pt);
                    emit_load(d, ov(a));
                    lhs = ov(d);
                }
            }
            continue;
        }
        if (match(TK_DOT)) {
            if (!at(TK_IDENT)) { perr(); return lhs; }
            Str member = peekv();
            advance();
            if (lhs.k == O_VAL) {
                Str n = vname(lhs);
                if (eq(n, "threadIdx") || eq(n, "blockIdx") || eq(n, "blockDim") || eq(n, "gridDim")) {
                    Str bi = cat(ar, n, S("."), member);
                    Str vn = cat(ar, n, S("_"), member);
                    uint32_t d = new_val(vn, S_UINT32);
                    Inst c = mk_inst(I_CALL, 0, (int32_t)d, onone(), onone());
                    c.func = bi;
                    emit(c);
                    lhs = ov(d);
                } else if (isstruct(lhs)) {
                    lhs = member_of_struct(lhs, member, src_name);
                } else if (isptr_struct(lhs)) {
                    lhs = member_of_ptr(lhs, member);
                }
            }
            continue;
        }
        if (match(TK_ARROW)) {
            if (!at(TK_IDENT)) { perr(); return lhs; }
            Str member = peekv();
            advance();
            if (isptr_struct(lhs)) lhs = member_of_ptr(lhs, member);
            continue;
        }
        break;
    }
    return lhs;
}

// Correctly rounded decimal -> double for literals the fast path covers
// (Clinger: <= 15 significant digits... up to 2^53, |exponent| <= 22).
OCB_HD inline bool parse_decimal_fast(Str s, double &out) {
    uint64_t mant = 0;
    int digits = 0, exp10 = 0;
    uint32_t i = 0;
    bool any = false;
    for (; i < s.n && s.p[i] >= '0' && s.p[i] <= '9'; ++i) {
        any = true;
        if (mant == 0 && s.p[i] == '0') continue;
        if (digits >= 19) return false;
        mant = mant * 10 + (s.p[i] - '0');
        ++digits;
    }
    if (i < s.n && s.p[i] == '.') {
        ++i;
        for (; i < s.n && s.p[i] >= '0' && s.p[i] <= '9'; ++i) {
            any = true;
            if (mant == 0 && s.p[i] == '0') { --exp10; continue; }
            if (digits >= 19) return false;
            mant = mant * 10 + (s.p[i] - '0');
            ++digits;
            --exp10;
        }
    }
    if (!any) return false;
    if (i < s.n && (s.p[i] == 'e' || s.p[i] == 'E')) {
        ++i;
        bool neg = false;
        if (i < s.n && (s.p[i] == '+' || s.p[i] == '-')) neg = s.p[i++] == '-';
        int e = 0;
        bool ed = false;
        for (; i < s.n && s.p[i] >= '0' && s.p[i] <= '9'; ++i) {
            ed = true;
            if (e < 100000) e = e * 10 + (s.p[i] - '0');
        }
        if (!ed) return false;
        exp10 += neg ? -e : e;
    }
    if (i != s.n) return false;
    if (mant == 0) { out = 0.0; return true; }
    if (mant > (1ull << 53) || exp10 < -22 || exp10 > 22) return false;
    const double p10[] = {1e0, 1e1, 1e2, 1e3, 1e4, 1e5, 1e6, 1e7, 1e8, 1e9, 1e10, 1e11,
                          1e12, 1e13, 1e14, 1e15, 1e16, 1e17, 1e18, 1e19, 1e20, 1e21, 1e22};
    double v = (double)mant;
    out = exp10 >= 0 ? v * p10[exp10] : v / p10[-exp10];
    return true;
}

// Exact decimal -> double, round half to even, for every literal the lexer
// accepts ([0-9]*.?[0-9]*([eE][+-]?[0-9]+)?): the value N * 10^E is formed
// with big integers (N: the significant digits, at most 60 of them), scaled
// by 2^s and divided by 10^-E when E < 0, then rounded to 53 bits or to the
// subnormal grid -- the result Python's float() gives.  Only literals the
// fast path above cannot take come here.
struct BigU {
    static constexpr int W = 56;   // 32-bit words: 1792 bits
    uint32_t w[W];
    int n;                         // words in use (no leading zero words)
    OCB_HD void set(uint32_t v) { n = v ? 1 : 0; w[0] = v; }
    OCB_HD bool mul_add(uint32_t m, uint32_t a) {
        uint64_t c = a;
        for (int i = 0; i < n; ++i) {
            uint64_t t = (uint64_t)w[i] * m + c;
            w[i] = (uint32_t)t;
            c = t >> 32;
        }
        if (c) {
            if (n >= W) return false;
            w[n++] = (uint32_t)c;
        }
        return true;
    }
    OCB_HD int bits() const {
        if (!n) return 0;
        uint32_t t = w[n - 1];
        int b = 0;
        while (t) { ++b; t >>= 1; }
        return (n - 1) * 32 + b;
    }
    OCB_HD bool bit(int i) const { return i >= 0 && i / 32 < n && ((w[i / 32] >> (i % 32)) & 1u); }
    OCB_HD bool any_below(int i) const {  // a set bit at a position < i
        for (int k = 0; k < n && k * 32 < i; ++k) {
            uint32_t m = (i - k * 32 >= 32) ? 0xFFFFFFFFu : ((1u << (i - k * 32)) - 1u);
            if (w[k] & m) return true;
        }
        return false;
    }
    OCB_HD uint64_t bits_from(int i, int cnt) const {  // cnt <= 54 bits starting at bit i
        uint64_t r = 0;
        for (int j = cnt - 1; j >= 0; --j) r = (r << 1) | (bit(i + j) ? 1u : 0u);
        return r;
    }
    OCB_HD bool shl1_or(uint32_t b) {
        uint32_t c = b;
        for (int i = 0; i < n; ++i) {
            uint32_t nc = w[i] >> 31;
            w[i] = (w[i] << 1) | c;
            c = nc;
        }
        if (c) {
            if (n >= W) return false;
            w[n++] = c;
        }
        return true;
    }
    OCB_HD int cmp(const BigU &o) const {
        if (n != o.n) return n < o.n ? -1 : 1;
        for (int i = n - 1; i >= 0; --i)
            if (w[i] != o.w[i]) return w[i] < o.w[i] ? -1 : 1;
        return 0;
    }
    OCB_HD void sub(const BigU &o) {  // *this -= o, *this >= o
        int64_t br = 0;
        for (int i = 0; i < n; ++i) {
            int64_t t = (int64_t)w[i] - (i < o.n ? o.w[i] : 0) - br;
            br = t < 0;
            w[i] = (uint32_t)(t + (br << 32));
        }
        while (n && !w[n - 1]) --n;
    }
};

OCB_HD inline bool parse_decimal_exact(Str s, double &out) {
    BigU N;
    N.set(0);
    int nd = 0, exp10 = 0;
    uint32_t i = 0;
    bool any = false, dot = false;
    for (; i < s.n; ++i) {
        char c = s.p[i];
        if (c == '.' && !dot) { dot = true; continue; }
        if (c < '0' || c > '9') break;
        any = true;
        if (dot) --exp10;
        if (nd == 0 && c == '0') continue;
        if (++nd > 60) return false;
        if (!N.mul_add(10, (uint32_t)(c - '0'))) return false;
    }
    if (!any) return false;
    if (i < s.n && (s.p[i] == 'e' || s.p[i] == 'E')) {
        ++i;
        bool neg = false;
        if (i < s.n && (s.p[i] == '+' || s.p[i] == '-')) neg = s.p[i++] == '-';
        int e = 0;
        bool ed = false;
        for (; i < s.n && s.p[i] >= '0' && s.p[i] <= '9'; ++i) {
            ed = true;
            if (e < 100000) e = e * 10 + (s.p[i] - '0');
        }
        if (!ed) return false;
        exp10 += neg ? -e : e;
    }
    if (i != s.n) return false;
    if (!N.n) { out = 0.0; return true; }
    if (exp10 + nd > 310) {  // beyond DBL_MAX: inf
        uint64_t inf_bits = 0x7FF0000000000000ull;
        memcpy(&out, &inf_bits, 8);
        return true;
    }
    if (exp10 + nd < -326) { out = 0.0; return true; }       // below half the least subnormal
    BigU Q;  // q = N * 10^E, or floor(N * 2^sh / 10^-E)
    int sh = 0;
    bool sticky = false;
    if (exp10 >= 0) {
        Q = N;
        for (int k = 0; k < exp10; ++k)
            if (!Q.mul_add(10, 0)) return false;
    } else {
        BigU D;
        D.set(1);
        for (int k = 0; k < -exp10; ++k)
            if (!D.mul_add(10, 0)) return false;
        sh = D.bits() - N.bits() + 56;
        if (sh < 0) sh = 0;
        // long division of N * 2^sh by D, one quotient bit at a time
        BigU R;
        R.set(0);
        Q.set(0);
        int nb = N.bits() + sh;
        for (int b = nb - 1; b >= 0; --b) {
            uint32_t nbit = (b >= sh && N.bit(b - sh)) ? 1u : 0u;
            if (!R.shl1_or(nbit)) return false;
            uint32_t qb = 0;
            if (R.cmp(D) >= 0) {
                R.sub(D);
                qb = 1;
            }
            if (!Q.shl1_or(qb)) return false;
        }
        sticky = R.n != 0;
    }
    // value = Q * 2^-sh (+ sticky); keep 53 bits or stop at 2^-1074
    int lq = Q.bits();
    int drop = lq - 53;
    if (drop < sh - 1074) drop = sh - 1074;
    uint64_t mant;
    if (drop <= 0) {
        mant = Q.bits_from(0, lq);
        out = ldexp((double)mant, -sh);
        return true;
    }
    mant = Q.bits_from(drop, lq - drop);
    bool half = Q.bit(drop - 1);
    bool rest = sticky || Q.any_below(drop - 1);
    if (half && (rest || (mant & 1))) ++mant;
    out = ldexp((double)mant, drop - sh);
    return true;
}

// float.fromhex of a hex-float literal without its [fFlL] suffix
// (lexer.py:282-284; the parser then reads back str() of it, the same
// double): 0x <hex digits> [. <hex digits>] p [+-] <decimal digits>, scaled
// by 2^exp and rounded half to even to 53 bits or to the subnormal grid.
// Values that overflow never get here (the lexer reports OverflowError).
OCB_HD inline bool parse_hexfloat(Str s, double &out) {
    uint32_t i = 0;
    if (s.n < 3 || s.p[0] != '0' || (s.p[1] | 0x20) != 'x') return false;
    i = 2;
    uint64_t m = 0;          // the first significant bits (up to 60)
    int mbits = 0;           // bits held in m
    int64_t scale = 0;       // value = m * 2^scale (+ sticky)
    bool sticky = false, dot = false, any = false;
    for (; i < s.n; ++i) {
        char c = s.p[i];
        if (c == '.' && !dot) { dot = true; continue; }
        uint32_t d;
        if (c >= '0' && c <= '9') d = c - '0';
        else if ((c | 0x20) >= 'a' && (c | 0x20) <= 'f') d = (c | 0x20) - 'a' + 10;
        else break;
        any = true;
        if (dot) scale -= 4;
        if (mbits + 4 <= 60) {
            m = (m << 4) | d;
            if (m) mbits += 4;
        } else {  // beyond 60 bits: keep the digit's weight, fold it into sticky
            scale += 4;
            sticky = sticky || d != 0;
        }
    }
    if (!any || i >= s.n || (s.p[i] | 0x20) != 'p') return false;
    ++i;
    bool neg = false;
    if (i < s.n && (s.p[i] == '+' || s.p[i] == '-')) neg = s.p[i++] == '-';
    int64_t e = 0;
    bool ed = false;
    for (; i < s.n && s.p[i] >= '0' && s.p[i] <= '9'; ++i) {
        ed = true;
        if (e < 100000) e = e * 10 + (s.p[i] - '0');
    }
    if (!ed || i != s.n) return false;
    scale += neg ? -e : e;
    if (m == 0) { out = 0.0; return true; }
#ifdef __CUDA_ARCH__
    int lq = 64 - __clzll((long long)m);
#else
    int lq = 64 - __builtin_clzll(m);
#endif
    int64_t drop = lq - 53;                       // bits below the 53 kept
    if (drop < -1074 - scale) drop = -1074 - scale;  // subnormal grid 2^-1074
    if (drop <= 0) {
        out = ldexp((double)m, (int)scale);
        return true;
    }
    if (drop > 63) { out = 0.0; return true; }    // far below the least subnormal
    uint64_t mant = m >> drop;
    bool half = (m >> (drop - 1)) & 1u;
    bool rest = sticky || (drop > 1 && (m & ((1ull << (drop - 1)) - 1)) != 0);
    if (half && (rest || (mant & 1))) ++mant;
    out = ldexp((double)mant, (int)(scale + drop));
    return true;
}

OCB_HD inline bool parse_decimal(Str s, double &out) {
    return parse_decimal_fast(s, out) || parse_decimal_exact(s, out);
}

// _parse_primary_expr (parser.py:1532-2249)
OCB_HD inline Opnd Parser::parse_primary_expr() {
    uint32_t k = peek();
    if (bad()) return onone();
    Str v = peekv();
    if (k == TK_CHAR_LIT) {
        advance();
        Str raw{v.p + 1, v.n >= 2 ? v.n - 2 : 0};
        int64_t iv = 0;
        if (raw.n >= 2 && raw.p[0] == '\\') {
            char e = raw.p[1];
            switch (e) {
            case 'n': iv = 10; break;
            case 't': iv = 9; break;
            case 'r': iv = 13; break;
            case '0': iv = 0; break;
            case '\\': iv = 92; break;
            case '\'': iv = 39; break;
            case '"': iv = 34; break;
            default: iv = (uint8_t)e;
            }
        } else {
            iv = raw.n ? (uint8_t)raw.p[0] : 0;
        }
        if (iv >= 0x80) unsup();
        return m.cint(S_INT32, iv);
    }
    if (k == TK_TRUE) { advance(); return m.cint(S_INT32, 1); }
    if (k == TK_FALSE) { advance(); return m.cint(S_INT32, 0); }
    if (k == TK_INT_LIT) {
        advance();
        uint32_t e = v.n;
        bool has_u = false, has_l = false;
        while (e > 0) {
            char c = v.p[e - 1] | 0x20;
            if (c == 'u') has_u = true;
            else if (c == 'l') has_l = true;
            else break;
            --e;
        }
        // int(stripped, 0) with C octal rewritten to 0o...
        pyint val = 0;
        uint32_t i = 0, base = 10;
        if (e >= 2 && v.p[0] == '0' && (v.p[1] | 0x20) == 'x') { base = 16; i = 2; }
        else if (e >= 2 && v.p[0] == '0' && (v.p[1] | 0x20) == 'b') { base = 2; i = 2; }
        else if (e >= 2 && v.p[0] == '0' && (v.p[1] | 0x20) == 'o') { base = 8; i = 2; }
        else if (e > 1 && v.p[0] == '0') { base = 8; i = 1; }
        if (i >= e) { raise_(R_VALUE); return onone(); }
        for (; i < e; ++i) {
            char c = v.p[i];
            uint32_t d = (c >= '0' && c <= '9') ? c - '0' : ((c | 0x20) >= 'a' && (c | 0x20) <= 'f') ? (c | 0x20) - 'a' + 10 : 99;
            if (d >= base) {  // int() rejects it: ValueError
                raise_(R_VALUE);
                return onone();
            }
            if (val > PYINT_LIM / 16) { unsup(); return onone(); }
            val = val * base + d;
        }
        Ty t;
        if (has_l || val > 0xFFFFFFFFll) t = has_u ? S_UINT64 : S_INT64;
        else if (has_u || val > 0x7FFFFFFFll) t = S_UINT32;
        else t = S_INT32;
        return m.cint(t, val);
    }
    if (k == TK_FLOAT_LIT) {
        advance();
        double d;
        if (v.n > 2 && v.p[0] == '0' && (v.p[1] | 0x20) == 'x') {  // hex float: [fFlL] suffix
            uint32_t e = v.n;
            while (e > 0 && ((v.p[e - 1] | 0x20) == 'f' || (v.p[e - 1] | 0x20) == 'l')) --e;
            if (!parse_hexfloat(Str{v.p, e}, d)) { unsup(); return onone(); }
            return m.cfloat(S_FLOAT, d);
        }
        uint32_t e = v.n;
        while (e > 0 && (v.p[e - 1] | 0x20) == 'f') --e;
        if (!parse_decimal(Str{v.p, e}, d)) { unsup(); return onone(); }
        return m.cfloat(S_FLOAT, d);
    }
    if (k == TK_IDENT || k == TK_HALF) {
        Str name = v;
        advance();
        while (at(TK_COLON) && pos + 1 < tk.n && kind_at(pos + 1) == TK_COLON) {
            advance();
            advance();
            if (at(TK_IDENT)) {
                name = peekv();
                advance();
            }
        }
        if (eq(name, "nullptr")) return m.cint(S_UINT64, 0);
        if ((eq(name, "static_cast") || eq(name, "reinterpret_cast") || eq(name, "const_cast")) &&
            at(TK_LT)) {
            // C++ named casts (parser.py:1610-1630): a type whose parse fails
            // (any exception) becomes INT32, each '*' wraps it in a global
            // pointer; a pointer operand in another space keeps its space
            advance();
            Ty ct;
            if (parse_type(ct)) {
                while (!bad() && match(TK_STAR)) {
                    bool ok = true;
                    ct = ty_ptr(ct, AS_GLOBAL, false, ok);
                    if (!ok) { unsup(); return onone(); }
                }
            }
            if (bad()) {
                if (!catch_any()) return onone();
                ct = S_INT32;
            }
            if (!expect(TK_GT) || !expect(TK_LPAREN)) return onone();
            Opnd opd = parse_assign_expr();
            if (bad() || !expect(TK_RPAREN)) return onone();
            if (is_ptr(ct) && opd.k == O_VAL && is_ptr(tyof(opd)) && ty_as(tyof(opd)) != AS_GLOBAL) {
                bool ok = true;
                ct = ty_ptr(ty_pointee(ct), ty_as(tyof(opd)), false, ok);
                if (!ok) { unsup(); return onone(); }
            }
            uint32_t d = new_val("cast", ct);
            emit_cvt(d, opd);
            return ov(d);
        }
        if (match(TK_LPAREN)) return parse_call(name);
        Opnd *vp = vars.get(name);
        if (vp) {
            Opnd var = *vp;
            if (shared_scalars.has(name) && var.k == O_VAL && is_ptr(tyof(var)) &&
                !at(TK_LBRACKET) && !at(TK_DOT)) {
                if (ty_is_struct(ty_pointee(tyof(var)))) {  // a whole-struct load
                    unsup();
                    return onone();
                }
                uint32_t d = new_val(name, ty_pointee(tyof(var)));
                emit_load(d, var);
                return ov(d);
            }
            return var;
        }
        if (Opnd *g = global_consts.get(name)) {
            if (g->k != O_SYM) return *g;
            // module variable (parser.py:2164-2185): its address before '[' and
            // for a non-scalar, else a load of the scalar through the symbol
            uint32_t gi = g->x;
            if (at(TK_LBRACKET) || !is_scalar_ty(m.gvars[gi].elem)) return gaddr(gi);
            uint32_t d = new_val(m.gvars[gi].name, m.gvars[gi].elem);
            emit_load(d, Opnd{O_SYM, gi});
            return ov(d);
        }
        if (eq(name, "true")) return m.cint(S_INT32, 1);
        if (eq(name, "false")) return m.cint(S_INT32, 0);
        if (eq(name, "NULL")) return m.cint(S_UINT64, 0);
        if (eq(name, "threadIdx") || eq(name, "blockIdx") || eq(name, "blockDim") ||
            eq(name, "gridDim"))
            return ov(m.add_val(0, S_INT32, name));  // placeholder, no id taken
        if (eq(name, "warpSize")) {
            uint32_t d = new_val("warpSize", S_UINT32);
            Inst c = mk_inst(I_CALL, 0, (int32_t)d, onone(), onone());
            c.func = S("warpSize");
            emit(c);
            return ov(d);
        }
        perr();
        return onone();
    }
    if (k == TK_STRING_LIT) { unsup(); return onone(); }
    if (k == TK_LPAREN) {
        advance();
        uint32_t pk = peek();
        bool type_ahead = pk == TK_VOID || pk == TK_INT || pk == TK_FLOAT || pk == TK_DOUBLE ||
                          pk == TK_HALF || pk == TK_CHAR || pk == TK_BOOL || pk == TK_SHORT ||
                          pk == TK_LONG || pk == TK_SIGNED || pk == TK_UNSIGNED ||
                          pk == TK_STRUCT || pk == TK_UNION || pk == TK_ENUM || pk == TK_CONST ||
                          pk == TK_VOLATILE;
        if (!type_ahead && pk == TK_IDENT && is_type_name(peekv())) type_ahead = true;
        if (type_ahead) {
            uint32_t saved = pos;
            Ty ct;
            bool ok = parse_type_with_ptr(ct);
            if (ok && at(TK_RPAREN)) {
                advance();
                if (at(TK_LBRACE) && ty_is_struct(ct)) return parse_compound_literal(ct);
                if (ty_is_struct(ct)) { unsup(); return onone(); }  // CvtInst to a struct
                Opnd o = parse_unary_expr();
                if (!bad()) {
                    uint32_t d = new_val("cast", ct);
                    emit_cvt(d, o);
                    return ov(d);
                }
            }
            if (bad()) {  // except Exception: self._pos = _saved
                if (!catch_any()) return onone();
                pos = saved;
            }
        }
        Opnd e = parse_expr();
        if (bad() || !expect(TK_RPAREN)) return e;
        return e;
    }
    perr();
    return onone();
}

// Built-in calls of _parse_primary_expr (parser.py:1635-2138) in the subset.
OCB_HD inline Opnd Parser::parse_call(Str name) {
    Vec<Opnd> args;
    args.init();
    bool is_printf = eq(name, "printf");
    // one argument; a printf argument that is one string literal is the
    // Const(VOID, 0) the reference's primary parser returns for it, its text
    // kept as the format (parser.py:2203-2209)
    auto arg = [&]() -> Opnd {
        if (is_printf && at(TK_STRING_LIT) && pos + 1 < tk.n &&
            (kind_at(pos + 1) == TK_COMMA || kind_at(pos + 1) == TK_RPAREN)) {
            last_string_lit = string_lit_text(peekv());
            advance();
            return m.cint(S_VOID, 0);
        }
        return parse_assign_expr();
    };
    if (!at(TK_RPAREN)) {
        args.push(ar, arg());
        while (!bad() && match(TK_COMMA)) args.push(ar, arg());
    }
    if (bad() || !expect(TK_RPAREN)) return onone();
    if (is_printf) {  // PrintfInst(fmt, args[1:]) (parser.py:1732-1738)
        Inst pi = mk_inst(I_PRINTF, 0, -1, onone(), onone());
        pi.func = last_string_lit;
        for (uint32_t q = 1; q < args.n; ++q) pi.args.push(ar, args[q]);
        emit(pi);
        return m.cint(S_VOID, 0);
    }
    auto call = [&](int32_t dest, Str func) {
        Inst c = mk_inst(I_CALL, 0, dest, onone(), onone());
        c.func = func;
        c.args = args;
        emit(c);
    };
    if (eq(name, "__syncthreads")) {
        call(-1, name);
        return m.cint(S_VOID, 0);
    }
    if (eq(name, "__all_sync") || eq(name, "__any_sync")) {
        uint32_t d = new_val(Str{name.p + 2, name.n - 2}, S_INT32);
        call((int32_t)d, name);
        return ov(d);
    }
    if (eq(name, "__shfl_sync") || eq(name, "__shfl_up_sync") || eq(name, "__shfl_down_sync") ||
        eq(name, "__shfl_xor_sync") || eq(name, "__ballot_sync")) {
        Ty rt = S_INT32;
        if (eq(name, "__ballot_sync")) rt = S_UINT32;
        else if (args.n > 1 && (args[1].k == O_VAL || args[1].k == O_CONST) && !is_ptr(tyof(args[1])))
            rt = tyof(args[1]);
        uint32_t d = new_val(Str{name.p + 2, name.n - 2}, rt);
        call((int32_t)d, name);
        return ov(d);
    }
    if (eq(name, "atomicAdd") || eq(name, "atomicSub") || eq(name, "atomicMin") ||
        eq(name, "atomicMax") || eq(name, "atomicAnd") || eq(name, "atomicOr") ||
        eq(name, "atomicXor") || eq(name, "atomicExch") || eq(name, "atomicCAS")) {
        if (args.n >= 2) {
            Ty rt = args[1].k == O_VAL ? tyof(args[1]) : (Ty)S_INT32;
            uint32_t d = new_val(cat(ar, S("atomic_"), name), rt);
            call((int32_t)d, name);
            return ov(d);
        }
        return m.cint(S_INT32, 0);
    }
    if (eq(name, "__ldg") || eq(name, "__ldcg") || eq(name, "__ldcs") || eq(name, "__ldlu") ||
        eq(name, "__ldca")) {
        if (args.n && args[0].k == O_VAL && is_ptr(tyof(args[0]))) {
            Ty pt = tyof(args[0]);
            if (eq(name, "__ldg")) {
                bool ok = true;
                Ty nct = ty_ptr(ty_pointee(pt), AS_CONST, false, ok);
                if (!ok) { unsup(); return onone(); }
                // Value(ptr.name, PtrTy(pointee, CONST), ptr.id): a second object, same id
                uint32_t nc = m.add_val(m.vals[args[0].x].id, nct, vname(args[0]));
                uint32_t d = new_val("ldg", ty_pointee(pt));
                emit_load(d, ov(nc));
                return ov(d);
            }
            uint32_t d = new_val(Str{name.p + 2, name.n - 2}, ty_pointee(pt));
            emit_load(d, args[0]);
            return ov(d);
        }
        return m.cint(S_INT32, 0);
    }
    // texture, surface and mbarrier intrinsics (parser.py:1645-1679)
    if (in_list(name, kTexFetch) || eq(name, "surf1Dread") || eq(name, "__mbarrier_try_wait_parity")) {
        uint32_t d = new_val(name, in_list(name, kTexFetch) ? (Ty)S_FLOAT : (Ty)S_INT32);
        call((int32_t)d, name);
        return ov(d);
    }
    if (in_list(name, kSurfVoid) || eq(name, "__mbarrier_init")) {
        call(-1, name);
        return m.cint(S_VOID, 0);
    }
    if (in_list(name, " __cp_async_bulk_tensor_1d __cp_async_bulk_tensor_2d"
                      " __cp_async_bulk_commit_group __cp_async_bulk_wait_group ")) {
        unsup();  // the bulk tensor copy intrinsics are not emitted by this engine
        return onone();
    }
    // recursive __device__ functions: a real call (parser.py:1739-1748)
    if (is_recursive(name)) {
        Ty rt = dfuncs[(uint32_t)find_dfunc(name)].ret;
        int32_t d = -1;
        if (!(ty_is_scalar(rt) && ty_scalar(rt) == S_VOID)) d = (int32_t)new_val(cat(ar, name, S("_ret")), rt);
        call(d, cat(ar, S("__devfn_"), name));
        return d >= 0 ? ov((uint32_t)d) : m.cint(S_VOID, 0);
    }
    // __device__ functions: expanded in place (parser.py:1749-1929)
    int32_t fi = find_dfunc(name);
    if (fi >= 0) return inline_call((uint32_t)fi, args, name);
    // generic intrinsic call (parser.py:1929-2138)
    if (in_list(name, kVoidStmts) || eq(name, "__syncwarp")) {
        call(-1, name);
        return m.cint(S_VOID, 0);
    }
    Ty rt = S_INT32;
    auto a0ty = [&](Ty dflt) -> Ty {
        return (args.n && (args[0].k == O_VAL || args[0].k == O_CONST)) ? tyof(args[0]) : dflt;
    };
    if (in_list(name, kSyncReduce)) rt = S_INT32;
    else if (eq(name, "__activemask")) rt = S_UINT32;
    else if (in_list(name, kIntOps)) rt = eq(name, "__brevll") ? (Ty)S_UINT64 : eq(name, "__brev") ? (Ty)S_UINT32 : (Ty)S_INT32;
    else if (eq(name, "clock64") || eq(name, "__clock64") || eq(name, "clock")) rt = contains(name, "64") ? S_UINT64 : S_UINT32;
    else if (in_list(name, kPredInt)) rt = S_INT32;
    else if (in_list(name, kFloat2Int)) rt = (contains(name, "ll") || contains(name, "longlong")) ? S_INT64 : S_INT32;
    else if (in_list(name, kInt2Float)) rt = contains(name, "double") ? S_DOUBLE : S_FLOAT;
    else if (eq(name, "__sad") || eq(name, "__usad")) rt = eq(name, "__usad") ? S_UINT32 : S_INT32;
    else if (in_list(name, " __dp4a __dp4a_u __dp4a_su __dp4a_us ")) rt = S_INT32;
    else if (in_list(name, kWarpReduceInt)) rt = S_INT32;
    else if (in_list(name, kWarpReduceUint) || eq(name, "__match_any_sync") || eq(name, "__match_all_sync")) rt = S_UINT32;
    else if (in_list(name, kIntBinary2)) rt = S_INT32;
    else if (in_list(name, kUintBinary2)) rt = S_UINT32;
    else if (in_list(name, kHalfUnary)) rt = (!eq(name, "__half2float") && !contains(name, "float")) ? S_HALF : S_FLOAT;
    else if (in_list(name, kHalfBinary) || in_list(name, kHalfTernary) || in_list(name, kHalfCvt)) rt = S_HALF;
    else if (in_list(name, kHalfCmpInt)) rt = S_INT32;
    else if (eq(name, "__half_as_ushort") || eq(name, "__half_as_short")) rt = S_UINT16;
    else if (in_list(name, kHalf2Int)) {
        if (contains(name, "ll")) rt = contains(name, "ull") ? S_UINT64 : S_INT64;
        else if (contains(name, "uint") || contains(name, "ushort")) rt = S_UINT32;
        else rt = S_INT32;
    } else if (eq(name, "__hadd") || eq(name, "__hadd_sat")) {
        Ty at = (args.n && args[0].k == O_VAL) ? tyof(args[0]) : (Ty)S_INT32;
        rt = at == S_HALF ? S_HALF : S_INT32;
    } else if (in_list(name, kFloatUnary) || in_list(name, kFloatBinary) || in_list(name, kFloatTernary)) {
        rt = a0ty(S_FLOAT) == S_DOUBLE ? S_DOUBLE : S_FLOAT;
    } else if (eq(name, "abs")) {
        rt = a0ty(S_INT32);
    } else if (eq(name, "min") || eq(name, "max")) {
        rt = args.n > 1 ? result_type(args[0], args[1]) : a0ty(S_INT32);
    }
    uint32_t d = new_val(name, rt);
    call((int32_t)d, name);
    return ov(d);
}

}  // namespace cc
}  // namespace ocb
