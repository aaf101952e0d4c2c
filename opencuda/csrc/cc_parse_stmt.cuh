// Parser, statements and top level: parser.py:2287-3705 (_parse_stmt,
// _parse_lvalue_or_expr, _parse_stmt_or_block), :3701-3874 (_parse_kernel)
// and :4194-4443 (parse_module), restated for the supported subset.
#pragma once
#include "cc_parse_devfn.cuh"

namespace ocb {
namespace cc {

OCB_HD inline bool is_decl_start_kind(uint32_t k) {
    return k == TK_INT || k == TK_UNSIGNED || k == TK_SIGNED || k == TK_FLOAT || k == TK_DOUBLE ||
           k == TK_VOID || k == TK_LONG || k == TK_HALF || k == TK_CHAR || k == TK_SHORT ||
           k == TK_BOOL || k == TK_STRUCT || k == TK_UNION || k == TK_ENUM;
}

// int(const.value) of an array dimension; floats are outside the subset
OCB_HD inline bool const_dim(Parser &P, Opnd o, int64_t &out) {
    if (o.k != O_CONST) {
        out = 1;
        return true;
    }
    const Const &c = P.m.consts[o.x];
    if (c.pyfloat || c.i > INT64_MAX / 2 || c.i < INT64_MIN / 2) {
        P.unsup();
        return false;
    }
    out = (int64_t)c.i;
    return true;
}

OCB_HD inline bool mul_dim(Parser &P, int64_t &size, int64_t d) {
    int64_t r;
    if (Parser::mul_ovf_(size, d, r)) {
        P.unsup();
        return false;
    }
    size = r;
    return true;
}

// _parse_lvalue_or_expr (parser.py:3414-3665)
OCB_HD inline Opnd Parser::parse_lvalue_or_expr() {
    uint32_t k = peek();
    if (bad()) return onone();
    if (k == TK_STAR && pos + 1 < tk.n && kind_at(pos + 1) == TK_IDENT) {
        Opnd *vp = vars.get(val_at(pos + 1));
        if (vp && is_ptr(tyof(*vp))) {
            pos += 2;
            return *vp;
        }
    }
    if (k == TK_IDENT) {
        Str name = peekv();
        Opnd *vp = vars.get(name);
        Opnd *gs = vp ? nullptr : global_consts.get(name);
        if (gs && gs->k == O_SYM && pos + 1 < tk.n) {
            // module variable as an lvalue: its address, or its element's
            // (parser.py:3433-3522)
            uint32_t nk = kind_at(pos + 1);
            if (nk == TK_ASSIGN || nk == TK_PLUS_EQ || nk == TK_MINUS_EQ || nk == TK_STAR_EQ ||
                nk == TK_SLASH_EQ || nk == TK_PERCENT_EQ || nk == TK_AMP_EQ || nk == TK_PIPE_EQ ||
                nk == TK_CARET_EQ || nk == TK_LSHIFT_EQ || nk == TK_RSHIFT_EQ || nk == TK_LBRACKET ||
                nk == TK_DOT) {
                uint32_t gi = gs->x;
                advance();
                Opnd addr = gaddr(gi);
                if (at(TK_LBRACKET)) {
                    advance();
                    Opnd index = parse_expr();
                    if (bad() || !expect(TK_RBRACKET)) return onone();
                    Ty gp = m.gvars[gi].ptr;
                    Opnd *rs = row_strides.get(m.gvars[gi].name);
                    if (rs && at(TK_LBRACKET)) {  // g[i][j]: row stride, then the element
                        Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                        uint32_t sc = new_val("scale", it);
                        emit_bin(sc, BO_MUL, index, m.cint(it, m.consts[rs->x].i));
                        uint32_t ra = new_val("raddr", gp);
                        emit_bin(ra, BO_ADD, addr, ov(sc));
                        advance();
                        Opnd col = parse_expr();
                        if (bad() || !expect(TK_RBRACKET)) return onone();
                        Ty et = ty_pointee(gp);
                        uint32_t ces = is_scalar_ty(et) ? ty_size(et) : 8;
                        if (ces != 1) {
                            Ty ct = isval(col) ? tyof(col) : (Ty)S_INT32;
                            uint32_t s2 = new_val("scale", ct);
                            emit_bin(s2, BO_MUL, col, m.cint(ct, ces));
                            col = ov(s2);
                        }
                        uint32_t ea = new_val("addr", gp);
                        emit_bin(ea, BO_ADD, ov(ra), col);
                        return field_chain(ov(ea), et, ty_as(gp));
                    }
                    uint32_t es = m.tsize(ty_pointee(gp));
                    if (es != 1) {
                        Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                        uint32_t sc = new_val("scale", it);
                        emit_bin(sc, BO_MUL, index, m.cint(it, es));
                        index = ov(sc);
                    }
                    uint32_t ea = new_val("addr", gp);
                    emit_bin(ea, BO_ADD, addr, index);
                    return field_chain(ov(ea), ty_pointee(gp), ty_as(gp));
                }
                Ty gp = m.gvars[gi].ptr;
                if (at(TK_DOT) && ty_is_struct(ty_pointee(gp)))  // g_struct.field = ...
                    return field_chain(addr, ty_pointee(gp), ty_as(gp));
                return addr;
            }
        }
        if (vp && is_ptr(tyof(*vp))) {
            Opnd var = *vp;
            Ty vt = tyof(var);
            advance();
            if ((at(TK_ARROW) || at(TK_DOT)) && ty_is_struct(ty_pointee(vt)))
                return member_lvalue(var);
            if (match(TK_LBRACKET)) {
                Opnd index = parse_expr();
                if (bad() || !expect(TK_RBRACKET)) return onone();
                Opnd addr;
                Opnd *rs = row_strides.get(name);
                if (rs && at(TK_LBRACKET)) {
                    Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                    uint32_t s = new_val("scale", it);
                    emit_bin(s, BO_MUL, index, m.cint(it, m.consts[rs->x].i));
                    uint32_t a = new_val("addr", vt);
                    emit_bin(a, BO_ADD, var, ov(s));
                    advance();
                    Opnd index2 = parse_expr();
                    if (bad() || !expect(TK_RBRACKET)) return onone();
                    uint32_t es = m.tsize(ty_pointee(vt));
                    if (es != 1) {
                        Ty it2 = isval(index2) ? tyof(index2) : (Ty)S_INT32;
                        uint32_t s2 = new_val("scale", it2);
                        emit_bin(s2, BO_MUL, index2, m.cint(it2, es));
                        index2 = ov(s2);
                    }
                    uint32_t f = new_val("addr", vt);
                    emit_bin(f, BO_ADD, ov(a), index2);
                    addr = ov(f);
                } else {
                    uint32_t es = m.tsize(ty_pointee(vt));
                    if (es != 1) {
                        Ty it = isval(index) ? tyof(index) : (Ty)S_INT32;
                        uint32_t s = new_val("scale", it);
                        emit_bin(s, BO_MUL, index, m.cint(it, es));
                        index = ov(s);
                    }
                    uint32_t a = new_val("addr", vt);
                    emit_bin(a, BO_ADD, var, index);
                    addr = ov(a);
                    Ty pt = ty_pointee(vt);
                    if (at(TK_LBRACKET) && is_ptr(pt)) {  // T**: load the row pointer
                        uint32_t rp = new_val("rowptr", pt);
                        emit_load(rp, addr);
                        advance();
                        Opnd index2 = parse_expr();
                        if (bad() || !expect(TK_RBRACKET)) return onone();
                        uint32_t es2 = m.tsize(ty_pointee(pt));
                        if (es2 != 1) {
                            Ty it2 = isval(index2) ? tyof(index2) : (Ty)S_INT32;
                            uint32_t s2 = new_val("scale", it2);
                            emit_bin(s2, BO_MUL, index2, m.cint(it2, es2));
                            index2 = ov(s2);
                        }
                        uint32_t f = new_val("addr", pt);
                        emit_bin(f, BO_ADD, ov(rp), index2);
                        addr = ov(f);
                    }
                }
                // p[i].pos.x = ...: chained fields stay addresses (parser.py:3645-3658)
                while (!bad() && at(TK_DOT) && isptr_struct(addr)) {
                    advance();
                    if (!at(TK_IDENT)) { perr(); return onone(); }
                    Str member = peekv();
                    advance();
                    addr = field_addr(addr, member);
                }
                return addr;
            }
            return var;
        }
    }
    return parse_expr();
}

OCB_HD inline void Parser::parse_stmt_or_block() {
    if (match(TK_LBRACE)) {
        VarMap outer = vars.copy(ar);
        NameSet ns;
        ns.init();
        scopes.push(ar, ns);
        while (!bad() && !match(TK_RBRACE)) parse_stmt();
        if (bad()) return;
        NameSet inner = scopes.back();
        scopes.n--;
        pop_scope(inner, outer);
    } else {
        parse_stmt();
    }
}

// End of a block scope: names declared inside either get their outer binding
// back or leave the map.  The reference walks a Python set, whose order only
// matters when two names are re-inserted at the end; that case is declined.
OCB_HD inline void Parser::pop_scope(NameSet &inner, VarMap &outer) {
    uint32_t reinserted = 0;
    for (uint32_t i = 0; i < inner.v.n; ++i) {
        Str name = inner.v[i];
        Opnd *o = outer.get(name);
        if (o) {
            if (!vars.has(name)) reinserted++;
            vars.set(ar, name, *o);
        } else if (vars.has(name)) {
            vars.del(ar, name);
        }
    }
    if (reinserted > 1) unsup();
}

// __shared__ declarations inside a kernel (parser.py:2377-2469)
OCB_HD inline void Parser::parse_shared(bool vol) {
    advance();
    Ty ty;
    if (!parse_type(ty)) return;
    if (!at(TK_IDENT)) { perr(); return; }
    Str name = peekv();
    advance();
    bool ok = true;
    Ty smem = ty_ptr(ty, AS_SHARED, vol, ok);
    if (!ok) { unsup(); return; }
    auto scalar = [&](Str n) {
        uint32_t v = new_val(n, smem);
        vars.set(ar, n, ov(v));
        shared_scalars.add(ar, n);
        kern->shared.push(ar, SharedDecl{n, ty, 1});
    };
    if (match(TK_SEMI)) {
        scalar(name);
        return;
    }
    if (at(TK_COMMA)) {
        scalar(name);
        while (!bad() && match(TK_COMMA)) {
            if (!at(TK_IDENT)) { perr(); return; }
            Str extra = peekv();
            advance();
            scalar(extra);
        }
        expect(TK_SEMI);
        return;
    }
    if (!expect(TK_LBRACKET)) return;
    if (at(TK_RBRACKET)) {  // extern __shared__ T name[]: dynamic, size 0
        advance();
        if (!expect(TK_SEMI)) return;
        uint32_t v = new_val(name, smem);
        vars.set(ar, name, ov(v));
        kern->shared.push(ar, SharedDecl{name, ty, 0});
        return;
    }
    auto array = [&](Str n, bool first) -> bool {
        if (!first) {
            if (!at(TK_IDENT)) { perr(); return false; }
            n = peekv();
            advance();
            if (!expect(TK_LBRACKET)) return false;
        }
        Opnd so = parse_assign_expr();
        if (bad()) return false;
        int64_t size;
        if (!const_dim(*this, so, size)) return false;
        if (!expect(TK_RBRACKET)) return false;
        int64_t inner = 1;
        bool has_inner = false;
        while (!bad() && at(TK_LBRACKET)) {
            advance();
            Opnd dop = parse_assign_expr();
            if (bad()) return false;
            int64_t d;
            if (!const_dim(*this, dop, d)) return false;
            has_inner = true;
            if (!mul_dim(*this, inner, d) || !mul_dim(*this, size, d)) return false;
            if (!expect(TK_RBRACKET)) return false;
        }
        if (bad()) return false;
        if (has_inner) {
            int64_t st = inner;
            if (!mul_dim(*this, st, is_scalar_ty(ty) ? ty_size(ty) : 8)) return false;
            row_strides.set(ar, n, m.cint(S_INT32, st));
        }
        uint32_t v = new_val(n, smem);
        vars.set(ar, n, ov(v));
        declare_local(n);
        kern->shared.push(ar, SharedDecl{n, ty, size});
        return true;
    };
    if (!array(name, true)) return;
    while (!bad() && match(TK_COMMA))
        if (!array(name, false)) return;
    if (!bad()) expect(TK_SEMI);
}

// Variable declarations (parser.py:2472-2741); `ty` is already parsed.
OCB_HD inline void Parser::parse_decl(Ty ty, bool) {
    for (;;) {
        Ty dty = ty;
        while (match(TK_STAR)) {
            bool ok = true;
            dty = ty_ptr(dty, AS_GLOBAL, false, ok);
            if (!ok) { unsup(); return; }
        }
        Str name;
        if (!expect_ident(name)) return;
        while (at(TK_IDENT) && eq(peekv(), "__attribute__")) {
            advance();
            if (at(TK_LPAREN)) {
                int depth = 1;
                advance();
                while (depth > 0 && !at(TK_EOF)) {
                    if (bad()) return;
                    uint32_t kk = peek();
                    if (kk == TK_LPAREN) depth++;
                    else if (kk == TK_RPAREN) depth--;
                    advance();
                }
            }
        }
        if (bad()) return;
        if (ty_is_struct(dty)) {  // struct / vector variable (parser.py:2502-2603)
            if (at(TK_LBRACKET)) {  // Foo arr[N]: .local, exposed as PtrTy(Foo, LOCAL)
                advance();
                Opnd so = parse_assign_expr();
                if (bad() || !expect(TK_RBRACKET)) return;
                int64_t count;
                if (!const_dim(*this, so, count)) return;
                bool ok = true;
                Ty aty = ty_ptr(dty, AS_LOCAL, false, ok);
                if (!ok) { unsup(); return; }
                uint32_t v = new_val(name, aty);
                vars.set(ar, name, ov(v));
                declare_local(name);
                kern->locals.push(ar, LocalDecl{name, dty, count, v});
                if (!match(TK_COMMA)) break;
                continue;
            }
            uint32_t sent = new_val(name, dty);
            vars.set(ar, name, ov(sent));
            declare_local(name);
            zero_init_fields(name, dty);
            if (bad()) return;
            if (match(TK_ASSIGN)) {
                if (at(TK_LBRACE)) {  // { e0, e1, ... } over the scalar fields
                    advance();
                    uint32_t nf = m.nfields(dty), fi = 0, i = 0;
                    while (!at(TK_RBRACE) && !at(TK_EOF)) {
                        if (bad()) return;
                        Opnd ve = parse_assign_expr();
                        if (bad()) return;
                        // the i-th scalar field
                        while (fi < nf && !is_scalar_ty(m.field(dty, fi).ty)) fi++;
                        if (fi < nf) {
                            SField f = m.field(dty, fi);
                            Str key = cat(ar, name, S("_"), f.name);
                            uint32_t fv = new_val(key, f.ty);
                            if (ve.k == O_CONST && m.consts[ve.x].ty != f.ty) {
                                Const c = m.consts[ve.x];
                                c.ty = f.ty;
                                m.consts.push(ar, c);
                                Opnd rc = oc(m.consts.n - 1);
                                uint32_t fv2 = new_val(key, f.ty);
                                emit_bin(fv2, BO_ADD, rc, m.czero(f.ty));
                                vars.set(ar, key, ov(fv2));
                            } else {
                                emit_bin(fv, BO_ADD, ve, m.czero(f.ty));
                                vars.set(ar, key, ov(fv));
                            }
                            fi++;
                        }
                        i++;
                        if (!match(TK_COMMA)) break;
                    }
                    (void)i;
                    if (bad() || !expect(TK_RBRACE)) return;
                } else {
                    Opnd rhs = parse_assign_expr();
                    if (bad()) return;
                    if (isptr_struct(rhs)) {  // Foo v = p[i]: load every field
                        load_struct_fields(rhs, ty_pointee(tyof(rhs)), name, 0,
                                           ty_as(tyof(rhs)), false, true);
                    } else if (isstruct(rhs)) {  // a struct value: copy its fields
                        uint32_t nf = m.nfields(dty);
                        for (uint32_t i = 0; i < nf && !bad(); ++i) {
                            SField f = m.field(dty, i);
                            if (!is_scalar_ty(f.ty)) continue;
                            Opnd src = struct_field_src(rhs.x, f.name);
                            if (src.k == O_NONE) continue;
                            Str key = cat(ar, name, S("_"), f.name);
                            uint32_t fv = new_val(key, f.ty);
                            emit_bin(fv, BO_ADD, src, m.czero(f.ty));
                            vars.set(ar, key, ov(fv));
                        }
                    }
                }
            }
            if (bad()) return;
            if (!match(TK_COMMA)) break;
            continue;
        }
        if (at(TK_LBRACKET)) {  // local array in .local
            advance();
            Opnd so = parse_assign_expr();
            if (bad() || !expect(TK_RBRACKET)) return;
            int64_t size;
            if (!const_dim(*this, so, size)) return;
            int64_t inner = 1;
            bool has_inner = false;
            while (!bad() && at(TK_LBRACKET)) {
                advance();
                Opnd dop = parse_assign_expr();
                if (bad()) return;
                int64_t d;
                if (!const_dim(*this, dop, d)) return;
                has_inner = true;
                if (!mul_dim(*this, inner, d) || !mul_dim(*this, size, d)) return;
                if (!expect(TK_RBRACKET)) return;
            }
            if (bad()) return;
            if (has_inner) {
                int64_t st = inner;
                if (!mul_dim(*this, st, is_scalar_ty(dty) ? ty_size(dty) : 8)) return;
                row_strides.set(ar, name, m.cint(S_INT32, st));
            }
            bool ok = true;
            Ty aty = ty_ptr(dty, AS_LOCAL, false, ok);
            if (!ok) { unsup(); return; }
            uint32_t v = new_val(name, aty);
            vars.set(ar, name, ov(v));
            declare_local(name);
            kern->locals.push(ar, LocalDecl{name, dty, size, v});
            if (match(TK_ASSIGN) && at(TK_LBRACE)) {
                advance();
                int64_t esz = is_scalar_ty(dty) ? ty_size(dty) : 8;
                int64_t idx = 0;
                // _emit_flat_elems: nested braces flatten into one element list.
                // State machine of the recursive walk; `depth` = open inner braces.
                int depth = 0;
                for (;;) {
                    if (bad()) return;
                    bool level_end = at(TK_RBRACE) || at(TK_EOF);
                    if (!level_end && at(TK_LBRACE)) {
                        advance();
                        if (++depth > MAX_NEST) { unsup(); return; }
                        continue;
                    }
                    if (!level_end) {
                        Opnd ev = parse_assign_expr();
                        if (bad()) return;
                        if (idx < size) {
                            uint32_t ea = new_val("earr", aty);
                            emit_bin(ea, BO_ADD, ov(v), m.cint(S_INT32, idx * esz));
                            if (ev.k == O_CONST && m.consts[ev.x].ty != dty) {
                                Const c = m.consts[ev.x];
                                c.ty = dty;
                                m.consts.push(ar, c);
                                ev = oc(m.consts.n - 1);
                            }
                            emit_store(ov(ea), ev);
                        }
                        idx++;
                        if (match(TK_COMMA)) continue;
                    }
                    // this level is done; close it and continue the parent level
                    bool finished = false;
                    for (;;) {
                        if (bad()) return;
                        if (depth == 0) { finished = true; break; }
                        if (!expect(TK_RBRACE)) return;
                        depth--;
                        if (match(TK_COMMA)) break;  // parent level goes on
                    }
                    if (finished) break;
                }
                if (!expect(TK_RBRACE)) return;
            }
            if (bad()) return;
            if (!match(TK_COMMA)) break;
            continue;
        }
        uint32_t v = new_val(name, dty);
        vars.set(ar, name, ov(v));
        declare_local(name);
        if (match(TK_ASSIGN)) {
            Opnd rhs = parse_assign_expr();
            if (bad()) return;
            vars.set(ar, name, rhs.k == O_VAL ? rhs : ov(v));
            if (rhs.k == O_CONST) {
                emit_bin(v, BO_ADD, rhs, m.cint(dty, 0));
                vars.set(ar, name, ov(v));
            } else if (rhs.k == O_VAL && !val_eq(rhs.x, v)) {
                Ty rt = tyof(rhs);
                if (is_scalar_ty(dty) && is_scalar_ty(rt) && dty != rt) {
                    emit_cvt(v, rhs);
                } else {
                    emit_bin(v, BO_ADD, rhs, m.cint(dty, 0));
                }
                vars.set(ar, name, ov(v));
            }
        } else {
            Opnd z = m.czero(dty);
            emit_bin(v, BO_ADD, z, z);
        }
        if (!match(TK_COMMA)) break;
    }
    if (!bad()) expect(TK_SEMI);
}

// if statement (parser.py:2743-2787)
OCB_HD inline void Parser::parse_if() {
    advance();
    if (!expect(TK_LPAREN)) return;
    Opnd c = parse_expr();
    if (bad() || !expect(TK_RPAREN)) return;
    uint32_t tb = new_block("if_true"), fb = new_block("if_false"), mb = new_block("if_merge");
    B().term = Term{T_CBR, c, m.blocks[tb].label, m.blocks[fb].label};
    VarMap before = vars.copy(ar);
    cur = tb;
    parse_stmt_or_block();
    if (bad()) return;
    loop_writeback(before);
    if (B().term.kind == T_NONE) B().term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
    vars = before.copy(ar);
    cur = fb;
    if (match(TK_ELSE)) {
        parse_stmt_or_block();
        if (bad()) return;
    }
    loop_writeback(before);
    if (B().term.kind == T_NONE) B().term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
    vars = before.copy(ar);
    cur = mb;
}

OCB_HD inline void Parser::push_loop(Str brk, Str cont, VarMap &snap) {
    break_targets.push(ar, brk);
    break_snaps.push(ar, snap);
    continue_targets.push(ar, cont);
    continue_snaps.push(ar, snap);
}
OCB_HD inline void Parser::pop_loop() {
    break_targets.n--;
    break_snaps.n--;
    continue_targets.n--;
    continue_snaps.n--;
}

// switch (parser.py:3030-3138): the case bodies are parsed in source order,
// each from the variables as they were before the switch; the dispatch is a
// compare chain built after the last case (switch_dispatch, switch_next_*),
// so its blocks and values come after every case block.  A switch pushes a
// break target only: `continue` still belongs to the enclosing loop.
OCB_HD inline void Parser::parse_switch() {
    advance();
    if (!expect(TK_LPAREN)) return;
    Opnd sv = parse_expr();
    if (bad() || !expect(TK_RPAREN) || !expect(TK_LBRACE)) return;
    uint32_t pre = cur;
    VarMap before = vars.copy(ar);
    uint32_t xb = new_block("switch_exit");
    break_targets.push(ar, m.blocks[xb].label);
    break_snaps.push(ar, before);
    Vec<Opnd> cvals;
    Vec<uint32_t> cblocks;
    cvals.init();
    cblocks.init();
    int32_t db = -1;       // default block
    int32_t fall = -1;     // block falling through into the next label
    while (!match(TK_RBRACE)) {
        if (bad()) return;
        uint32_t k = peek();
        if (bad()) return;
        if (k == TK_CASE || k == TK_DEFAULT) {
            if (B().term.kind == T_NONE && cur != pre) {
                loop_writeback(before);
                fall = (int32_t)cur;
            } else {
                fall = -1;
            }
            uint32_t nb;
            if (k == TK_CASE) {
                advance();
                Opnd cv = parse_expr();
                if (bad() || !expect(TK_COLON)) return;
                nb = new_block("case");
                cvals.push(ar, cv);
                cblocks.push(ar, nb);
            } else {
                advance();
                if (!expect(TK_COLON)) return;
                nb = new_block("default");
                db = (int32_t)nb;
            }
            if (fall >= 0) {
                m.blocks[fall].term = Term{T_BR, onone(), m.blocks[nb].label, Str{nullptr, 0}};
                fall = -1;
            }
            vars = before.copy(ar);
            cur = nb;
        } else {
            parse_stmt();
        }
        if (bad()) return;
    }
    break_targets.n--;
    break_snaps.n--;
    Str xl = m.blocks[xb].label;
    if (B().term.kind == T_NONE) {
        loop_writeback(before);
        B().term = Term{T_BR, onone(), xl, Str{nullptr, 0}};
    }
    for (uint32_t q = 0; q < cblocks.n; ++q) {
        if (m.blocks[cblocks[q]].term.kind == T_NONE) {
            cur = cblocks[q];
            loop_writeback(before);
            B().term = Term{T_BR, onone(), xl, Str{nullptr, 0}};
        }
    }
    if (db >= 0 && m.blocks[db].term.kind == T_NONE) {
        cur = (uint32_t)db;
        loop_writeback(before);
        B().term = Term{T_BR, onone(), xl, Str{nullptr, 0}};
    }
    uint32_t eb = new_block("switch_dispatch");
    if (m.blocks[pre].term.kind == T_NONE)
        m.blocks[pre].term = Term{T_BR, onone(), m.blocks[eb].label, Str{nullptr, 0}};
    uint32_t c = eb;
    for (uint32_t q = 0; q < cblocks.n && !bad(); ++q) {
        uint32_t d = new_val("cmp", S_BOOL);
        cur = c;
        emit_cmp(d, CO_EQ, sv, cvals[q]);
        uint32_t nx = new_block("switch_next");
        m.blocks[c].term = Term{T_CBR, ov(d), m.blocks[cblocks[q]].label,
                                m.blocks[nx].label};
        c = nx;
    }
    cur = c;
    B().term = Term{T_BR, onone(), db >= 0 ? m.blocks[db].label : xl, Str{nullptr, 0}};
    vars = before.copy(ar);
    cur = xb;
}

// for loop (parser.py:2789-2900)
OCB_HD inline void Parser::parse_for() {
    advance();
    if (!expect(TK_LPAREN)) return;
    VarMap for_outer = vars.copy(ar);
    NameSet ns;
    ns.init();
    scopes.push(ar, ns);
    parse_stmt();  // init
    if (bad()) return;
    uint32_t cond_start = pos;
    int depth = 0;
    for (;;) {
        uint32_t kk = peek();
        if (bad()) return;
        if (kk == TK_SEMI && depth == 0) break;
        if (kk == TK_LPAREN) depth++;
        if (kk == TK_RPAREN) depth--;
        advance();
    }
    advance();
    uint32_t inc_start = pos;
    depth = 0;
    for (;;) {
        uint32_t kk = peek();
        if (bad()) return;
        if (kk == TK_RPAREN && depth == 0) break;
        if (kk == TK_LPAREN) depth++;
        if (kk == TK_RPAREN) depth--;
        advance();
    }
    if (!expect(TK_RPAREN)) return;
    uint32_t body_resume = pos;
    VarMap loop_vars = vars.copy(ar);
    uint32_t cb = new_block("for_cond"), bb = new_block("for_body"), ib = new_block("for_inc"),
             eb = new_block("for_exit");
    B().term = Term{T_BR, onone(), m.blocks[cb].label, Str{nullptr, 0}};
    cur = cb;
    pos = cond_start;
    Opnd c;
    if (kind_at(cond_start) == TK_SEMI) {
        c = m.cint(S_INT32, 1);
    } else {
        c = parse_expr();
        if (bad()) return;
    }
    B().term = Term{T_CBR, c, m.blocks[bb].label, m.blocks[eb].label};
    pos = body_resume;
    cur = bb;
    push_loop(m.blocks[eb].label, m.blocks[ib].label, loop_vars);
    parse_stmt_or_block();
    if (bad()) return;
    pop_loop();
    if (B().term.kind == T_NONE) {
        loop_writeback(loop_vars);
        B().term = Term{T_BR, onone(), m.blocks[ib].label, Str{nullptr, 0}};
    }
    cur = ib;
    uint32_t saved = pos;
    pos = inc_start;
    if (kind_at(inc_start) != TK_RPAREN) {
        parse_assign_expr();
        while (!bad() && match(TK_COMMA)) parse_assign_expr();
        if (bad()) return;
    }
    pos = saved;
    for (uint32_t i = 0; i < loop_vars.e.n; ++i) {
        const VarEnt &en = loop_vars.e[i];
        if (!en.live || en.v.k != O_VAL) continue;
        Opnd *cv = vars.get(en.name);
        if (!cv || (cv->k == O_VAL && cv->x == en.v.x)) continue;
        if (cv->k == O_VAL) {
            emit_bin(en.v.x, BO_ADD, *cv, m.cint(tyof(en.v), 0));
            vars.set(ar, en.name, en.v);
        }
    }
    B().term = Term{T_BR, onone(), m.blocks[cb].label, Str{nullptr, 0}};
    cur = eb;
    NameSet inner = scopes.back();
    scopes.n--;
    pop_scope(inner, for_outer);
}

// while and do/while loops (parser.py:2902-2998)
OCB_HD inline void Parser::parse_while() {
    advance();
    if (!expect(TK_LPAREN)) return;
    VarMap entry = vars.copy(ar);
    uint32_t cb = new_block("while_cond"), bb = new_block("while_body"),
             eb = new_block("while_exit");
    B().term = Term{T_BR, onone(), m.blocks[cb].label, Str{nullptr, 0}};
    cur = cb;
    Opnd c = parse_expr();
    if (bad() || !expect(TK_RPAREN)) return;
    B().term = Term{T_CBR, c, m.blocks[bb].label, m.blocks[eb].label};
    cur = bb;
    push_loop(m.blocks[eb].label, m.blocks[cb].label, entry);
    parse_stmt_or_block();
    if (bad()) return;
    pop_loop();
    loop_writeback(entry);
    if (B().term.kind == T_NONE) B().term = Term{T_BR, onone(), m.blocks[cb].label, Str{nullptr, 0}};
    cur = eb;
}

OCB_HD inline void Parser::parse_do() {
    advance();
    VarMap entry = vars.copy(ar);
    uint32_t bb = new_block("do_body"), cb = new_block("do_cond"), eb = new_block("do_exit");
    B().term = Term{T_BR, onone(), m.blocks[bb].label, Str{nullptr, 0}};
    cur = bb;
    push_loop(m.blocks[eb].label, m.blocks[cb].label, entry);
    parse_stmt_or_block();
    if (bad()) return;
    pop_loop();
    loop_writeback(entry);
    if (B().term.kind == T_NONE) B().term = Term{T_BR, onone(), m.blocks[cb].label, Str{nullptr, 0}};
    cur = cb;
    if (!expect(TK_WHILE) || !expect(TK_LPAREN)) return;
    Opnd c = parse_expr();
    if (bad() || !expect(TK_RPAREN) || !expect(TK_SEMI)) return;
    B().term = Term{T_CBR, c, m.blocks[bb].label, m.blocks[eb].label};
    cur = eb;
}

// Expression statement (parser.py:3186-3412)
OCB_HD inline void Parser::parse_expr_stmt() {
    Str stmt_lhs{nullptr, 0};
    if (at(TK_IDENT)) {
        Str cand = peekv();
        uint32_t np = pos + 1;
        if (np < tk.n) {
            uint32_t nk = kind_at(np);
            if ((nk == TK_ASSIGN || nk == TK_PLUS_EQ || nk == TK_MINUS_EQ || nk == TK_STAR_EQ) &&
                vars.has(cand))
                stmt_lhs = cand;
        }
    }
    if (bad()) return;
    Opnd lhs = parse_lvalue_or_expr();
    if (bad()) return;
    if (match(TK_ASSIGN)) {
        Opnd rhs = parse_expr();
        if (bad()) return;
        if (isval(lhs) && is_ptr(tyof(lhs))) {
            if (stmt_lhs.p && shared_scalars.has(stmt_lhs)) stmt_lhs = Str{nullptr, 0};
            Str un = stmt_lhs.p ? stmt_lhs : vname(lhs);
            if (stmt_lhs.p && vars.has(un)) {
                vars.set(ar, un, rhs);
            } else if (isstruct(rhs) && ty_is_struct(ty_pointee(tyof(lhs)))) {
                // *p = s / a[i] = s: one store per scalar field (parser.py:3258-3274)
                Ty st = ty_pointee(tyof(lhs));
                uint32_t as = ty_as(tyof(lhs));
                uint32_t nf = m.nfields(st);
                for (uint32_t i = 0; i < nf && !bad(); ++i) {
                    SField f = m.field(st, i);
                    if (!is_scalar_ty(f.ty)) continue;
                    Opnd fv = struct_field_src(rhs.x, f.name);
                    if (fv.k == O_NONE) continue;
                    bool ok = true;
                    Ty fp = ty_ptr(f.ty, as, false, ok);
                    if (!ok) { unsup(); return; }
                    uint32_t fa = new_val("faddr", fp);
                    emit_bin(fa, BO_ADD, lhs, m.cint(S_INT32, m.field_offset(st, i)));
                    emit_store(ov(fa), fv);
                }
            } else {
                Ty pt = ty_pointee(tyof(lhs));
                if (isval(rhs) && is_scalar_ty(tyof(rhs)) && is_scalar_ty(pt) && tyof(rhs) != pt) {
                    uint32_t co = new_val("coerce", pt);
                    emit_cvt(co, rhs);
                    rhs = ov(co);
                }
                emit_store(lhs, rhs);
            }
        } else if (isval(lhs)) {
            Str un = stmt_lhs.p ? stmt_lhs : vname(lhs);
            Opnd *pp = vars.get(un);
            if (pp) {
                Opnd prev = *pp;
                if (isval(rhs) && prev.k == O_VAL && is_scalar_ty(tyof(prev)) &&
                    is_scalar_ty(tyof(rhs)) && !eq(vname(rhs), un)) {
                    Ty pt = tyof(prev);
                    uint32_t mat = new_val(un, pt);
                    emit_bin(mat, BO_ADD, rhs, m.czero(pt));
                    rhs = ov(mat);
                }
                vars.set(ar, un, rhs);
                if (isstruct(rhs)) copy_struct_fields(rhs.x, un);
            }
        }
        while (!bad() && match(TK_COMMA)) {
            Str l2name{nullptr, 0};
            if (at(TK_IDENT)) l2name = peekv();
            Opnd l2 = parse_lvalue_or_expr();
            if (bad()) return;
            if (match(TK_ASSIGN)) {
                Opnd r2 = parse_assign_expr();
                if (bad()) return;
                if (isval(l2) && !is_ptr(tyof(l2))) {
                    Str u2 = l2name.p ? l2name : vname(l2);
                    if (vars.has(u2)) vars.set(ar, u2, r2);
                }
            }
        }
        if (!bad()) expect(TK_SEMI);
        return;
    }
    static const uint32_t toks[] = {TK_PLUS_EQ, TK_MINUS_EQ, TK_STAR_EQ, TK_SLASH_EQ,
                                    TK_PERCENT_EQ, TK_AMP_EQ, TK_PIPE_EQ, TK_CARET_EQ,
                                    TK_LSHIFT_EQ, TK_RSHIFT_EQ};
    static const uint8_t ops[] = {BO_ADD, BO_SUB, BO_MUL, BO_DIV, BO_MOD,
                                  BO_AND, BO_OR, BO_XOR, BO_SHL, BO_SHR};
    for (int kx = 0; kx < 10; ++kx) {
        if (!match(toks[kx])) continue;
        uint8_t op = ops[kx];
        Opnd rhs = parse_expr();
        if (bad()) return;
        if (isval(lhs) && is_ptr(tyof(lhs))) {
            Ty lt = tyof(lhs);
            bool is_ptr_var = stmt_lhs.p && vars.has(stmt_lhs) && !shared_scalars.has(stmt_lhs);
            if (is_ptr_var && (op == BO_ADD || op == BO_SUB)) {
                Opnd sc = scale_ptr_off(lt, rhs);
                if (bad()) return;
                uint32_t r = new_val("compound", lt);
                emit_bin(r, op, lhs, sc);
                vars.set(ar, stmt_lhs, ov(r));
            } else {
                uint32_t cv = new_val("cur", ty_pointee(lt));
                emit_load(cv, lhs);
                uint32_t r = new_val("compound", ty_pointee(lt));
                emit_bin(r, op, ov(cv), rhs);
                emit_store(lhs, ov(r));
            }
        } else {
            uint32_t r = new_val("compound", isval(lhs) ? tyof(lhs) : (Ty)S_INT32);
            emit_bin(r, op, lhs, rhs);
            Str un = stmt_lhs.p ? stmt_lhs : (isval(lhs) ? vname(lhs) : Str{nullptr, 0});
            if (un.p && vars.has(un)) vars.set(ar, un, ov(r));
        }
        expect(TK_SEMI);
        return;
    }
    for (int kx = 0; kx < 2; ++kx) {
        if (!match(kx == 0 ? TK_PLUSPLUS : TK_MINUSMINUS)) continue;
        uint8_t op = kx == 0 ? BO_ADD : BO_SUB;
        if (isval(lhs)) {
            Ty lt = tyof(lhs);
            if (is_ptr(lt)) {
                Str un = stmt_lhs.p ? stmt_lhs : vname(lhs);
                bool is_ptr_var = vars.has(un) && !shared_scalars.has(un);
                if (is_ptr_var) {
                    Ty pt = ty_pointee(lt);
                    int64_t step = is_scalar_ty(pt) ? ty_size(pt) : 1;
                    uint32_t np = new_val(cat(ar, vname(lhs), S("_inc")), lt);
                    emit_bin(np, op, lhs, m.cint(S_UINT64, step));
                    vars.set(ar, un, ov(np));
                } else {
                    Ty pt = ty_pointee(lt);
                    uint32_t cv = new_val("cur", pt);
                    emit_load(cv, lhs);
                    uint32_t r = new_val("compound", pt);
                    emit_bin(r, op, ov(cv), m.cint(pt, 1));
                    emit_store(lhs, ov(r));
                }
            } else {
                uint32_t nv = new_val(cat(ar, vname(lhs), S("_inc")), lt);
                emit_bin(nv, op, lhs, m.cint(lt, 1));
                Str un = stmt_lhs.p ? stmt_lhs : vname(lhs);
                if (vars.has(un)) vars.set(ar, un, ov(nv));
            }
        }
        expect(TK_SEMI);
        return;
    }
    while (!bad() && match(TK_COMMA)) parse_assign_expr();
    if (!bad()) expect(TK_SEMI);
}

// asm [volatile] ("template" : "=r"(out), ... : "r"(expr), ... : clobbers);
// (parser.py:2326-2375): each output names a variable that gets a fresh value
// of its old type (int when unbound); the template is kept as written.
OCB_HD inline void Parser::parse_asm() {
    advance();
    if (at(TK_VOLATILE) || (at(TK_IDENT) && eq(peekv(), "volatile"))) advance();
    if (!expect(TK_LPAREN)) return;
    Str tmpl{"", 0};
    if (at(TK_STRING_LIT)) {
        Str v = peekv();
        tmpl = Str{v.p + 1, v.n >= 2 ? v.n - 2 : 0};
        advance();
    }
    Vec<Opnd> outs, ins;
    outs.init();
    ins.init();
    if (match(TK_COLON)) {
        while (at(TK_STRING_LIT)) {
            advance();
            if (!expect(TK_LPAREN)) return;
            if (!at(TK_IDENT)) { perr(); return; }
            Str vn = peekv();
            advance();
            if (!expect(TK_RPAREN)) return;
            Opnd *old = vars.get(vn);
            Ty t = old ? tyof(*old) : (Ty)S_INT32;
            uint32_t nv = new_val(vn, t);
            outs.push(ar, ov(nv));
            vars.set(ar, vn, ov(nv));
            if (!match(TK_COMMA)) break;
        }
        if (bad()) return;
        if (match(TK_COLON)) {
            while (at(TK_STRING_LIT)) {
                advance();
                if (!expect(TK_LPAREN)) return;
                Opnd e = parse_assign_expr();
                if (bad() || !expect(TK_RPAREN)) return;
                ins.push(ar, e);
                if (!match(TK_COMMA)) break;
            }
            if (bad()) return;
            if (match(TK_COLON)) {
                while (at(TK_STRING_LIT)) {
                    advance();
                    if (!match(TK_COMMA)) break;
                }
            }
        }
    }
    if (bad() || !expect(TK_RPAREN) || !expect(TK_SEMI)) return;
    if (!tmpl.n) return;
    Inst ai = mk_inst(I_ASM, 0, -1, onone(), onone());
    ai.func = tmpl;
    ai.pidx = outs.n;
    for (uint32_t q = 0; q < outs.n; ++q) ai.args.push(ar, outs[q]);
    for (uint32_t q = 0; q < ins.n; ++q) ai.args.push(ar, ins[q]);
    emit(ai);
}

// _parse_stmt (parser.py:2287-3412)
OCB_HD inline void Parser::parse_stmt() {
    if (++nest > MAX_NEST) { unsup(); --nest; return; }
    parse_stmt_inner();
    --nest;
}

OCB_HD inline void Parser::parse_stmt_inner() {
    uint32_t k = peek();
    bool vol = false;
    while (k == TK_CONST || k == TK_VOLATILE || k == TK_STATIC) {
        if (k == TK_VOLATILE) vol = true;
        advance();
        k = peek();
    }
    if (bad()) return;
    if (k == TK_SEMI) { advance(); return; }
    if (k == TK_GOTO) {
        advance();
        if (at(TK_IDENT)) advance();
        match(TK_SEMI);
        return;
    }
    if (k == TK_IDENT && pos + 1 < tk.n && kind_at(pos + 1) == TK_COLON) {
        pos += 2;  // label: a no-op
        return;
    }
    if (k == TK_LBRACE) { parse_stmt_or_block(); return; }
    if (k == TK_IDENT) {
        Str v = peekv();
        if (eq(v, "asm") || eq(v, "__asm__") || eq(v, "__asm")) { parse_asm(); return; }
    }
    if (k == TK_SHARED) { parse_shared(vol); return; }
    bool decl = is_decl_start_kind(k);
    if (!decl && k == TK_IDENT) decl = is_type_name(peekv());
    if (decl) {
        Ty ty;
        if (!parse_type_with_ptr(ty)) return;
        parse_decl(ty, vol);
        return;
    }
    switch (k) {
    case TK_IF: parse_if(); return;
    case TK_FOR: parse_for(); return;
    case TK_WHILE: parse_while(); return;
    case TK_DO: parse_do(); return;
    case TK_SWITCH: parse_switch(); return;
    case TK_BREAK:
    case TK_CONTINUE: {
        bool brk = k == TK_BREAK;
        advance();
        if (!expect(TK_SEMI)) return;
        Vec<Str> &tg = brk ? break_targets : continue_targets;
        Vec<VarMap> &sn = brk ? break_snaps : continue_snaps;
        if (!tg.n) { perr(); return; }
        if (sn.n) loop_writeback(sn.back());
        B().term = Term{T_BR, onone(), tg.back(), Str{nullptr, 0}};
        cur = new_block(brk ? "after_break" : "after_continue");
        return;
    }
    case TK_RETURN: {
        advance();
        Opnd rv = onone();
        if (at(TK_SEMI)) {
            advance();
        } else {
            rv = parse_expr();
            if (bad() || !expect(TK_SEMI)) return;
        }
        if (inline_dest >= 0) {  // inside an inlined __device__ body (parser.py:3150-3189)
            Ty dt = m.vals[inline_dest].ty;
            if (rv.k != O_NONE && ty_is_struct(dt) && isstruct(rv)) {
                // struct result: copies into the canonical field values
                uint32_t rid = m.vals[inline_dest].id;
                uint32_t nf = m.nfields(dt);
                for (uint32_t q = 0; q < nf && !bad(); ++q) {
                    SField fd = m.field(dt, q);
                    if (!is_scalar_ty(fd.ty)) continue;
                    Opnd src = struct_field_src(rv.x, fd.name);
                    if (src.k == O_NONE) continue;
                    int32_t e = isrf_find(rid, fd.name);
                    uint32_t df;
                    if (e >= 0) {
                        df = isrf[e].v.x;
                    } else {
                        df = new_val(cat(ar, m.vals[inline_dest].name, S("_"), fd.name), fd.ty);
                        isrf_set(rid, fd.name, ov(df));
                    }
                    emit_bin(df, BO_ADD, src, m.czero(fd.ty));
                }
            } else if (rv.k != O_NONE && (ty_is_struct(dt) || isstruct(rv))) {
                unsup();  // a struct copied as one value: no PTX for it
                return;
            } else if (rv.k != O_NONE)
                emit_bin((uint32_t)inline_dest, BO_ADD, rv, m.czero(m.vals[inline_dest].ty));
            B().term = Term{T_BR, onone(), inline_merge, Str{nullptr, 0}};
            cur = new_block("after_inline_return");
            return;
        }
        B().term = Term{T_RET, rv, Str{nullptr, 0}, Str{nullptr, 0}};
        return;
    }
    default: break;
    }
    parse_expr_stmt();
}

OCB_HD inline bool is_fn_qualifier(Str v) {
    return eq(v, "__launch_bounds__") || eq(v, "__attribute__") || eq(v, "__noinline__") ||
           eq(v, "__forceinline__") || eq(v, "__inline__");
}

// int(token.value) of a __launch_bounds__ argument: decimal digits only
OCB_HD inline bool py_int_decimal(Str s, int64_t &out) {
    if (!s.n || s.n > 18) return false;
    int64_t v = 0;
    for (uint32_t i = 0; i < s.n; ++i) {
        if (s.p[i] < '0' || s.p[i] > '9') return false;
        v = v * 10 + (s.p[i] - '0');
    }
    out = v;
    return true;
}

// _parse_kernel (parser.py:3701-3874)
OCB_HD inline void Parser::parse_kernel() {
    if (!expect(TK_GLOBAL)) return;
    int64_t lb[2];
    bool lb_set[2] = {false, false};
    auto skip_qual = [&]() {
        Str qn = peekv();
        advance();
        if (!at(TK_LPAREN)) return;
        advance();
        if (eq(qn, "__launch_bounds__")) {
            uint32_t kk = peek();
            if (kk == TK_INT_LIT || kk == TK_IDENT) {
                int64_t v;
                if (py_int_decimal(peekv(), v)) { lb[0] = v; lb_set[0] = true; }
                else if (kk == TK_INT_LIT && peekv().n > 18) unsup();
                advance();
                if (match(TK_COMMA)) {
                    kk = peek();
                    if (kk == TK_INT_LIT || kk == TK_IDENT) {
                        if (py_int_decimal(peekv(), v)) { lb[1] = v; lb_set[1] = true; }
                        else if (kk == TK_INT_LIT && peekv().n > 18) unsup();
                        advance();
                    }
                }
            }
        }
        int depth = 1;
        while (depth > 0) {
            uint32_t kk = peek();
            if (bad()) return;
            if (kk == TK_LPAREN) depth++;
            if (kk == TK_RPAREN) depth--;
            advance();
        }
    };
    while (!bad() && at(TK_IDENT) && is_fn_qualifier(peekv())) skip_qual();
    Ty rt;
    if (bad() || !parse_type(rt)) return;
    while (!bad() && at(TK_IDENT) && is_fn_qualifier(peekv())) skip_qual();
    if (bad()) return;
    if (!at(TK_IDENT)) { perr(); return; }
    Str name = peekv();
    advance();
    if (!expect(TK_LPAREN)) return;
    Vec<Param> params;
    params.init();
    if (at(TK_VOID) && kind_at(pos + 1) == TK_RPAREN) advance();
    if (bad()) return;
    if (!at(TK_RPAREN)) {
        for (;;) {
            Ty pty;
            if (!parse_type_with_ptr(pty)) return;
            Str pname;
            if (!expect_ident(pname)) return;
            if (at(TK_LBRACKET)) {  // array parameter: PtrTy(ty, 0) (parser.py:3768-3774)
                advance();
                while (!at(TK_RBRACKET)) {
                    if (bad()) return;
                    if (at(TK_EOF)) { unsup(); return; }  // the reference never returns
                    advance();
                }
                advance();
                if (!is_ptr(pty)) {
                    bool ok = true;
                    pty = ty_ptr(pty, AS_INT0, false, ok);
                    if (!ok) { unsup(); return; }
                }
            }
            while (at(TK_IDENT) && eq(peekv(), "__attribute__")) {
                advance();
                if (at(TK_LPAREN)) {
                    int depth = 1;
                    advance();
                    while (depth > 0 && !at(TK_EOF)) {
                        if (bad()) return;
                        uint32_t kk = peek();
                        if (kk == TK_LPAREN) depth++;
                        else if (kk == TK_RPAREN) depth--;
                        advance();
                    }
                }
            }
            if (bad()) return;
            params.push(ar, Param{pname, pty});
            if (!match(TK_COMMA)) break;
        }
    }
    if (bad() || !expect(TK_RPAREN)) return;
    Kernel kk;
    kk.name = name;
    kk.params = params;
    kk.blocks.init();
    kk.next_id = 0;
    kk.n_launch = 0;
    if (lb_set[0]) {
        kk.launch[kk.n_launch++] = lb[0];
        if (lb_set[1]) kk.launch[kk.n_launch++] = lb[1];
    }
    kk.shared.init();
    kk.locals.init();
    kk.has_locals = false;
    kk.ret = S_VOID;
    if (!m.kernels.push(ar, kk)) return;  // arena exhausted
    kern = &m.kernels.back();
    kidx = m.kernels.n - 1;
    vars.init();
    block_count = 0;
    isrf.init();
    copy_src.init();
    uint32_t entry = new_block("entry");
    cur = entry;
    NameSet seen;
    seen.init();
    for (uint32_t i = 0; i < params.n; ++i) {
        if (ty_is_struct(params[i].ty)) {  // flattened to one ParamInst per leaf field
            if (!vars.has(params[i].name)) {
                uint32_t sv = new_val(params[i].name, params[i].ty);
                vars.set(ar, params[i].name, ov(sv));
            }
            uint32_t next;
            flat_struct_params(params[i].name, params[i].ty, i, seen, next);
            if (bad()) return;
            continue;
        }
        if (seen.has(params[i].name)) continue;
        uint32_t v = new_val(params[i].name, params[i].ty);
        Inst pi = mk_inst(I_PARAM, 0, (int32_t)v, onone(), onone());
        pi.pidx = i;
        pi.func = params[i].name;
        emit(pi);
        vars.set(ar, params[i].name, ov(v));
        seen.add(ar, params[i].name);
    }
    for (uint32_t i = 0; i < module_shared.n; ++i) {
        bool ok = true;
        Ty st = ty_ptr(module_shared[i].ty, AS_SHARED, false, ok);
        if (!ok) { unsup(); return; }
        uint32_t v = new_val(module_shared[i].name, st);
        vars.set(ar, module_shared[i].name, ov(v));
        kern->shared.push(ar, SharedDecl{module_shared[i].name, module_shared[i].ty,
                                         module_shared[i].count});
    }
    if (!expect(TK_LBRACE)) return;
    while (!bad() && !match(TK_RBRACE)) parse_stmt();
    if (bad()) return;
    if (B().term.kind == T_NONE) B().term = Term{T_RET, onone(), Str{nullptr, 0}, Str{nullptr, 0}};
}

// enum (parser.py:3944-3972): enumerators become module-level INT32
// constants, folded at parse time; the tag names INT32.
OCB_HD inline void Parser::parse_enum_def() {
    if (!expect(TK_ENUM)) return;
    if (at(TK_IDENT)) {
        add_typedef(peekv(), S_INT32);
        advance();
    }
    if (!expect(TK_LBRACE)) return;
    pyint counter = 0;
    while (!at(TK_RBRACE)) {
        if (bad()) return;
        if (!at(TK_IDENT)) {
            perr();
            return;
        }
        Str name = peekv();
        advance();
        if (match(TK_ASSIGN)) {
            Opnd v = parse_assign_expr();
            if (bad()) return;
            counter = 0;  // a non-constant initializer counts as 0
            if (v.k == O_CONST) {
                const Const &c = m.consts[v.x];
                if (c.pyfloat) {  // int(float): truncation
                    if (!(c.f == c.f) || c.f >= 1e30 || c.f <= -1e30) {
                        unsup();
                        return;
                    }
                    counter = (pyint)c.f;
                } else {
                    counter = c.i;
                }
            }
        }
        global_consts.set(ar, name, m.cint(S_INT32, counter));
        counter += 1;
        if (!py_ok(counter)) {
            unsup();
            return;
        }
        if (!match(TK_COMMA)) break;
    }
    if (bad() || !expect(TK_RBRACE)) return;
    match(TK_SEMI);
}

// typedef (parser.py:3974-4029): scalar, pointer, struct and union aliases,
// enum aliases, function-pointer and array typedefs (the alias names the
// return / element type).
OCB_HD inline void Parser::parse_typedef() {
    if (!expect(TK_TYPEDEF)) return;
    if (at(TK_ENUM)) {
        parse_enum_def();
        if (bad()) return;
        if (at(TK_IDENT)) {
            add_typedef(peekv(), S_INT32);
            advance();
        }
        match(TK_SEMI);
        return;
    }
    if (at(TK_STRUCT) || at(TK_UNION)) {  // typedef struct [Tag] { ... } Alias;
        Ty st;
        if (!parse_struct_def(st)) return;
        if (at(TK_IDENT)) {
            add_typedef(peekv(), st);
            advance();
            match(TK_SEMI);
        } else {
            add_typedef(m.structs[ty_sidx(st)].name, st);
        }
        return;
    }
    Ty ty;
    if (!parse_type_with_ptr(ty)) return;
    if (at(TK_LPAREN)) {  // ret_ty (*alias)(params...)
        advance();
        match(TK_STAR);
        bool named = at(TK_IDENT);
        Str alias = named ? peekv() : Str{nullptr, 0};
        if (named) advance();
        match(TK_RPAREN);
        if (at(TK_LPAREN)) {
            int depth = 0;
            while (!at(TK_EOF)) {
                uint32_t kk = peek();
                advance();
                if (kk == TK_LPAREN) {
                    depth++;
                } else if (kk == TK_RPAREN) {
                    if (--depth == 0) break;
                }
            }
        }
        match(TK_SEMI);
        if (named) add_typedef(alias, ty);
        return;
    }
    if (!at(TK_IDENT)) {
        perr();
        return;
    }
    Str alias = peekv();
    advance();
    if (at(TK_LBRACKET)) {  // typedef T name[N]: the dimension is parsed and dropped
        advance();
        if (!at(TK_RBRACKET)) {
            parse_assign_expr();
            if (bad()) return;
        }
        if (!expect(TK_RBRACKET)) return;
    }
    if (!expect(TK_SEMI)) return;
    add_typedef(alias, ty);
}

// __device__ function definition (parser.py:4031-4087): signature, then the
// body is skipped and kept as a token range for inlining.
OCB_HD inline void Parser::parse_device_func() {
    if (!expect(TK_DEVICE)) return;
    while (at(TK_DEVICE) || at(TK_STATIC) ||
           (at(TK_IDENT) && in_list(peekv(), " __noinline__ __forceinline__ __inline__ "
                                             "__attribute__ __cdecl__ __stdcall__ __fastcall__ ")))
        advance();
    if (bad()) return;
    Ty rt;
    if (!parse_type_with_ptr(rt)) return;
    if (!at(TK_IDENT)) {
        perr();
        return;
    }
    Str name = peekv();
    advance();
    if (!expect(TK_LPAREN)) return;
    Vec<Param> params;
    params.init();
    if (at(TK_VOID) && kind_at(pos + 1) == TK_RPAREN) advance();
    if (bad()) return;
    if (!at(TK_RPAREN)) {
        for (;;) {
            Ty pty;
            if (!parse_type_with_ptr(pty)) return;
            Str pname;
            if (!expect_ident(pname)) return;
            if (at(TK_LBRACKET)) {  // array parameter: PtrTy(ty, 0) (parser.py:4051-4059)
                advance();
                while (!at(TK_RBRACKET)) {
                    if (bad()) return;
                    if (at(TK_EOF)) { unsup(); return; }  // the reference never returns
                    advance();
                }
                advance();
                if (!is_ptr(pty)) {
                    bool ok = true;
                    pty = ty_ptr(pty, AS_INT0, false, ok);
                    if (!ok) { unsup(); return; }
                }
            }
            params.push(ar, Param{pname, pty});
            if (!match(TK_COMMA)) break;
        }
    }
    if (bad() || !expect(TK_RPAREN)) return;
    if (match(TK_SEMI)) return;  // a prototype registers nothing
    uint32_t bs = pos;
    if (!expect(TK_LBRACE)) return;
    int depth = 1;
    while (depth > 0) {
        uint32_t kk = peek();
        if (bad()) return;
        if (kk == TK_EOF) {  // unterminated body: the reference never returns
            unsup();
            return;
        }
        if (kk == TK_LBRACE) depth++;
        if (kk == TK_RBRACE) depth--;
        advance();
    }
    dfuncs.push(ar, DevFunc{name, rt, params, bs, pos});
}

// Call of a __device__ function (parser.py:1749-1929, scalar form): the
// arguments bind the parameter names, the body is parsed again in place with
// `return` writing `<name>_ret` and branching to `inline_<name>_merge`, and
// the caller's variables are restored afterwards.
OCB_HD inline Opnd Parser::inline_call(uint32_t fi, Vec<Opnd> &args, Str name) {
    if (inline_depth >= 16) {
        unsup();
        return onone();
    }
    DevFunc f = dfuncs[fi];
    VarMap saved_vars = vars.copy(ar);
    uint32_t saved_pos = pos;
    int32_t saved_dest = inline_dest;
    Str saved_merge = inline_merge;
    // caller variables passed as &x: reloaded from their slot afterwards
    struct Spilled {
        Str name;
        Ty ty;
        Opnd slot;
    };
    Vec<Spilled> spilled;
    spilled.init();
    for (uint32_t k = 0; k < args.n; ++k) {
        Opnd a = args[k];
        if (a.k != O_VAL || !is_ptr(tyof(a)) || ty_as(tyof(a)) != AS_LOCAL) continue;
        for (uint32_t q = 0; q < saved_vars.e.n; ++q) {
            const VarEnt &ve = saved_vars.e[q];
            if (!ve.live || !starts(ve.name, "_spill_") || ve.v.k != O_VAL ||
                m.vals[ve.v.x].id != m.vals[a.x].id)
                continue;
            Str orig = Str{ve.name.p + 7, ve.name.n - 7};
            Opnd *ov0 = saved_vars.get(orig);
            if (ov0 && ov0->k == O_VAL) spilled.push(ar, Spilled{orig, tyof(*ov0), a});
            break;
        }
    }
    for (uint32_t k = 0; k < f.params.n && k < args.n && !bad(); ++k) {
        Str pn = f.params[k].name;
        Ty pty = f.params[k].ty;
        Opnd a = args[k];
        if (ty_is_struct(pty) && a.k == O_VAL) {
            // a fresh sentinel named after the parameter; its fields are the
            // argument's (loaded through a struct pointer, or the caller's
            // `<arg>_<field>` values) (parser.py:1790-1853)
            uint32_t ps = new_val(pn, pty);
            vars.set(ar, pn, ov(ps));
            if (isptr_struct(a)) {
                load_struct_fields(a, ty_pointee(tyof(a)), pn, 0, ty_as(tyof(a)), true, true);
            } else {
                uint32_t nf = m.nfields(pty);
                for (uint32_t q = 0; q < nf; ++q) {
                    SField fd = m.field(pty, q);
                    if (ty_is_struct(fd.ty)) continue;
                    Opnd *cf = vars.get(cat(ar, vname(a), S("_"), fd.name));
                    if (cf) {
                        Opnd cv = *cf;
                        vars.set(ar, cat(ar, pn, S("_"), fd.name), cv);
                    }
                }
            }
        } else {
            vars.set(ar, pn, a);
        }
    }
    uint32_t rd = new_val(cat(ar, name, S("_ret")), f.ret);
    uint32_t mb = new_block(cat(ar, S("inline_"), name, S("_merge")));
    if (bad()) return onone();
    inline_dest = (int32_t)rd;
    inline_merge = m.blocks[mb].label;
    if (ty_is_struct(f.ret)) {  // one canonical value per scalar field of the result
        uint32_t nf = m.nfields(f.ret);
        for (uint32_t q = 0; q < nf && !bad(); ++q) {
            SField fd = m.field(f.ret, q);
            if (!is_scalar_ty(fd.ty)) continue;
            uint32_t fv = new_val(cat(ar, m.vals[rd].name, S("_"), fd.name), fd.ty);
            isrf_set(m.vals[rd].id, fd.name, ov(fv));
        }
    }
    Vec<NameSet> saved_scopes = scopes;
    scopes.init();
    ++inline_depth;
    pos = f.body_start;
    if (!expect(TK_LBRACE)) return onone();
    while (!at(TK_RBRACE)) {
        if (bad()) return onone();
        parse_stmt();
        if (bad()) return onone();
    }
    advance();
    --inline_depth;
    if (B().term.kind == T_NONE) B().term = Term{T_BR, onone(), m.blocks[mb].label, Str{nullptr, 0}};
    cur = mb;
    pos = saved_pos;
    vars = saved_vars;
    for (uint32_t k = 0; k < spilled.n && !bad(); ++k) {
        Ty sty = spilled[k].ty;
        if (ty_is_struct(sty)) {  // reload every scalar / pointer field of the slot
            uint32_t nf = m.nfields(sty);
            for (uint32_t q = 0; q < nf && !bad(); ++q) {
                SField fd = m.field(sty, q);
                if (ty_is_struct(fd.ty)) continue;
                bool ok = true;
                Ty fp = ty_ptr(fd.ty, AS_LOCAL, false, ok);
                if (!ok) { unsup(); return onone(); }
                uint32_t fa = new_val("faddr", fp);
                emit_bin(fa, BO_ADD, spilled[k].slot, m.cint(S_INT32, m.field_offset(sty, q)));
                Str key = cat(ar, spilled[k].name, S("_"), fd.name);
                uint32_t u = new_val(key, fd.ty);
                emit_load(u, ov(fa));
                vars.set(ar, key, ov(u));
            }
            continue;
        }
        uint32_t u = new_val(spilled[k].name, spilled[k].ty);
        emit_load(u, spilled[k].slot);
        vars.set(ar, spilled[k].name, ov(u));
    }
    inline_dest = saved_dest;
    inline_merge = saved_merge;
    scopes = saved_scopes;
    // the result's field values, visible as `<name>_ret_<field>`
    uint32_t rid = m.vals[rd].id;
    for (uint32_t q = 0; q < isrf.n && !bad(); ++q)
        if (isrf[q].vid == rid) {
            Opnd fv = isrf[q].v;
            vars.set(ar, cat(ar, m.vals[rd].name, S("_"), isrf[q].fname), fv);
        }
    return ov(rd);
}

// parse_module (parser.py:4194-4437): pass 1 registers module-level names and
// records kernel positions; pass 2 parses the kernels in order.
// A module-level variable: `__device__ [static] [__constant__] [volatile] T
// name[N] [= init];` (parser.py:4305-4366) or `__constant__ [const|static|
// __device__]* T name[N] [= init];` (parser.py:4155-4191).  The initializer is
// skipped, as there; the name is bound to a symbol in the same table as the
// module's enum constants, and the variable joins the module's declarations.
OCB_HD inline void Parser::parse_gvar(bool constant_form) {
    bool is_const = constant_form, is_vol = false;
    if (constant_form) {
        advance();  // __constant__
        while (at(TK_CONST) || at(TK_STATIC) || at(TK_DEVICE)) advance();
    } else {
        while (at(TK_DEVICE) || at(TK_STATIC)) advance();
        if (at(TK_CONSTANT)) {
            is_const = true;
            advance();
        }
        if (at(TK_VOLATILE)) {
            is_vol = true;
            advance();
        }
    }
    Ty t;
    if (!parse_type_with_ptr(t)) return;
    if (!constant_form && is_ptr(t) && ty_vol(t)) is_vol = true;
    if (!at(TK_IDENT)) { perr(); return; }
    Str name = peekv();
    advance();
    int64_t count = 1;
    if (match(TK_LBRACKET)) {
        Opnd so = parse_assign_expr();
        if (bad()) return;
        if (!const_dim(*this, so, count)) return;
        if (!expect(TK_RBRACKET)) return;
        // further dimensions of a __device__ array multiply the count and give
        // the row stride its element-address lvalues use (parser.py:4334-4348);
        // the __constant__ form reads one dimension and leaves the rest to the
        // module loop, which skips it token by token
        if (!constant_form && at(TK_LBRACKET)) {
            int64_t inner = 1;
            while (at(TK_LBRACKET) && !bad()) {
                advance();
                Opnd dop = parse_assign_expr();
                if (bad()) return;
                int64_t dim;
                if (!const_dim(*this, dop, dim)) return;
                if (!mul_dim(*this, count, dim) || !mul_dim(*this, inner, dim)) return;
                if (!expect(TK_RBRACKET)) return;
            }
            int64_t es = is_scalar_ty(t) ? (int64_t)ty_size(t) : 8;
            if (!mul_dim(*this, inner, es)) return;
            row_strides.set(ar, name, m.cint(S_INT32, inner));
        }
    }
    if (count > 0x7fffffff || count < -0x7fffffff) { unsup(); return; }
    if (match(TK_ASSIGN)) {  // skip the initializer
        int depth = 0;
        while (!at(TK_EOF) && !bad()) {
            uint32_t kk = peek();
            if (kk == TK_LBRACE) {
                depth++;
                advance();
            } else if (kk == TK_RBRACE) {
                depth--;
                advance();
                if (depth == 0) break;
            } else if (depth == 0 && kk == TK_SEMI) {
                break;
            } else {
                advance();
            }
        }
    }
    match(TK_SEMI);
    uint32_t sp = is_const ? AS_CONST : AS_GLOBAL;
    bool ok = true;
    Ty pt = ty_ptr(t, sp, is_vol, ok);
    if (!ok) { unsup(); return; }
    if (!m.gvars.push(ar, GVar{name, t, pt, (uint32_t)(int32_t)count, sp})) { unsup(); return; }
    global_consts.set(ar, name, Opnd{O_SYM, m.gvars.n - 1});
}

// GlobalAddrInst(Value(f"{sym}_ptr", sym.ty), sym, space)
OCB_HD inline Opnd Parser::gaddr(uint32_t g) {
    const GVar &gv = m.gvars[g];
    uint32_t d = new_val(cat(ar, gv.name, S("_ptr")), gv.ptr);
    Inst in{};
    in.kind = I_GADDR;
    in.op = (uint8_t)gv.space;
    in.dest = (int32_t)d;
    in.func = gv.name;
    emit(in);
    return ov(d);
}

OCB_HD inline void Parser::parse_module() {
    if (bad() || !m.vals.cap || !m.blocks.cap || !m.insts.cap || !m.consts.cap) {
        ar.oom = true;
        return;
    }
    Vec<uint32_t> kpos;
    kpos.init();
    while (!bad() && !at(TK_EOF)) {
        while (at(TK_STATIC)) advance();
        if (bad()) return;
        if (at(TK_CONST)) {
            uint32_t saved = pos;
            advance();
            Ty t;
            bool done = false;
            if (parse_type_with_ptr(t)) {
                if (at(TK_IDENT)) {
                    Str name = peekv();
                    advance();
                    if (match(TK_ASSIGN)) {
                        Opnd vo = parse_assign_expr();
                        if (!bad()) {
                            if (vo.k == O_CONST) global_consts.set(ar, name, vo);
                            while (!at(TK_SEMI) && !at(TK_EOF)) advance();
                            match(TK_SEMI);
                            done = true;
                        }
                    }
                }
            }
            if (done) continue;
            if (bad() && !catch_any()) return;
            pos = saved;
        }
        if (bad()) return;
        if (at(TK_IDENT) && eq(peekv(), "namespace")) {
            advance();
            if (at(TK_IDENT)) advance();
            if (at(TK_LBRACE)) advance();
            continue;
        }
        if (at(TK_IDENT) && eq(peekv(), "template")) {
            advance();
            if (at(TK_LT)) {
                advance();
                int depth = 1;
                while (depth > 0 && !at(TK_EOF)) {
                    uint32_t kk = peek();
                    if (kk == TK_LT) depth++;
                    else if (kk == TK_GT) depth--;
                    advance();
                }
            }
            continue;
        }
        uint32_t k = peek();
        if (k == TK_GLOBAL) {
            uint32_t la = pos + 1;
            bool fwd = false;
            while (la < tk.n) {
                uint32_t lk = kind_at(la);
                if (lk == TK_LBRACE) break;
                if (lk == TK_SEMI) { fwd = true; break; }
                la++;
            }
            if (fwd) {
                while (!at(TK_SEMI) && !at(TK_EOF)) advance();
                if (at(TK_SEMI)) advance();
            } else {
                kpos.push(ar, pos);
                while (!at(TK_LBRACE) && !at(TK_EOF)) advance();
                if (at(TK_LBRACE)) {
                    int depth = 1;
                    advance();
                    while (depth > 0 && !at(TK_EOF)) {
                        uint32_t kk = peek();
                        if (kk == TK_LBRACE) depth++;
                        else if (kk == TK_RBRACE) depth--;
                        advance();
                    }
                }
            }
        } else if (k == TK_TYPEDEF) {
            parse_typedef();
        } else if (k == TK_ENUM) {
            parse_enum_def();
        } else if (k == TK_DEVICE) {
            // a function when '(' comes before ';' (parser.py:4282-4304)
            bool is_func = false;
            for (uint32_t la = pos + 1; la < tk.n; ++la) {
                uint32_t lk = kind_at(la);
                if (lk == TK_LPAREN) {
                    is_func = true;
                    break;
                }
                if (lk == TK_SEMI || lk == TK_EOF) break;
            }
            if (!is_func) {
                parse_gvar(false);
                continue;
            }
            parse_device_func();
        } else if (k == TK_CONSTANT) {
            parse_gvar(true);
        } else if (k == TK_STRUCT || k == TK_UNION) {
            Ty st;
            parse_struct_def(st);
        } else if (k == TK_SHARED) {
            advance();
            Ty t;
            if (!parse_type(t)) return;
            if (!at(TK_IDENT)) { perr(); return; }
            Str name = peekv();
            advance();
            if (!expect(TK_LBRACKET)) return;
            int64_t count = 0;
            if (!at(TK_RBRACKET)) {
                Opnd so = parse_assign_expr();
                if (bad()) return;
                if (!const_dim(*this, so, count)) return;
            }
            if (!expect(TK_RBRACKET)) return;
            match(TK_SEMI);
            module_shared.push(ar, SharedInit{name, t, count});
        } else {
            advance();
        }
    }
    if (bad()) return;
    // recursion detection, then each recursive function compiled as a .func
    // in the order of the reference's set (parser.py:4392-4435)
    if (!recursive_funcs(rec_funcs)) {
        unsup();
        return;
    }
    for (uint32_t i = 0; i < rec_funcs.n && !bad(); ++i) compile_devfn(rec_funcs[i]);
    for (uint32_t i = 0; i < kpos.n && !bad(); ++i) {
        pos = kpos[i];
        parse_kernel();
    }
}

}  // namespace cc
}  // namespace ocb
