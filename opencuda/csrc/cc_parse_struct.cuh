// Parser, structs and unions: the StructTy paths of opencuda/frontend/parser.py
// (struct definitions :3876-3942, the built-in vector types :98-128, member
// access :1388-1530, declarations :2502-2603, struct-to-struct copies
// :642-668 and :3322-3348, compound literals :2251-2283, kernel parameter
// flattening :3801-3846).
//
// A struct variable is never one value: the reference keeps a *sentinel*
// Value of StructTy under the variable's name (for type lookups) and one SSA
// value per scalar field under `<name>_<field>` in the variable map.  Those
// keys, the sentinels' value ids and the order of every emitted instruction
// are visible in the output (value ids become register numbers), so these
// routines follow the reference step by step.
#pragma once
#include "cc_parse_expr.cuh"

namespace ocb {
namespace cc {

// The CUDA vector types, registered as StructTy (parser.py:112-128).
OCB_HD inline bool Parser::vector_type(Str v, Ty &t) {
    struct VT {
        const char *name;
        uint32_t base;
        uint32_t n;
    };
    static const VT tbl[20] = {
        {"float2", S_FLOAT, 2},  {"float3", S_FLOAT, 3},  {"float4", S_FLOAT, 4},
        {"double2", S_DOUBLE, 2}, {"int2", S_INT32, 2},   {"int3", S_INT32, 3},
        {"int4", S_INT32, 4},    {"uint2", S_UINT32, 2},  {"uint3", S_UINT32, 3},
        {"uint4", S_UINT32, 4},  {"short2", S_INT32, 2},  {"ushort2", S_UINT32, 2},
        {"char2", S_INT32, 2},   {"uchar2", S_UINT32, 2}, {"char4", S_INT32, 4},
        {"uchar4", S_UINT32, 4}, {"long2", S_INT64, 2},   {"ulong2", S_UINT64, 2},
        {"longlong2", S_INT64, 2}, {"ulonglong2", S_UINT64, 2}};
    if (v.n < 4 || v.n > 10) return false;
    for (int i = 0; i < 20; ++i) {
        if (!eq(v, tbl[i].name)) continue;
        if (!vec_types[i]) {
            static const char *const names[4] = {"x", "y", "z", "w"};
            SField f[4];
            for (uint32_t j = 0; j < tbl[i].n; ++j) f[j] = SField{S(names[j]), tbl[i].base};
            vec_types[i] = m.add_struct(S(tbl[i].name), f, tbl[i].n);
        }
        t = vec_types[i];
        return true;
    }
    return false;
}

OCB_HD inline bool Parser::is_type_name(Str v) {
    Ty t;
    return user_typedef(v, t) || typedef_scalar(v, t) || vector_type(v, t) || user_struct(v, t);
}

OCB_HD inline uint32_t Parser::field_array(Ty st, Str member) {
    Str sn = m.structs[ty_sidx(st)].name;
    uint32_t group = 0xFFFFFFFFu;
    for (uint32_t i = farrs.n; i-- > 0;)
        if (eq(farrs[i].sname, sn)) {
            group = farrs[i].group;
            break;
        }
    if (group == 0xFFFFFFFFu) return 0;
    for (uint32_t i = farrs.n; i-- > 0;)
        if (farrs[i].group == group && eq(farrs[i].base, member)) return farrs[i].count;
    return 0;
}

// _parse_struct_def (parser.py:3876-3942)
OCB_HD inline bool Parser::parse_struct_def(Ty &out) {
    if (!match(TK_STRUCT) && !expect(TK_UNION)) return false;
    Str name;
    if (at(TK_IDENT)) {
        name = peekv();
        advance();
    } else {
        name = cat(ar, S("__anon_"), utoa(ar, block_count));
        block_count++;
    }
    if (bad()) return false;
    if (!at(TK_LBRACE)) {  // a use without a body
        if (find_struct(name, out)) return true;
        perr();
        return false;
    }
    advance();
    Vec<SField> fields;
    fields.init();
    uint32_t group = farr_groups++;
    bool any_arr = false;
    while (!at(TK_RBRACE)) {
        if (bad()) return false;
        if (at(TK_IDENT) && pos + 1 < tk.n && kind_at(pos + 1) == TK_COLON) {
            Str a = peekv();
            if (eq(a, "public") || eq(a, "private") || eq(a, "protected")) {
                pos += 2;
                continue;
            }
        }
        Ty fty;
        if (!parse_type_with_ptr(fty)) return false;
        for (;;) {
            if (!at(TK_IDENT)) {
                perr();
                return false;
            }
            Str fname = peekv();
            advance();
            int64_t count = 1;
            while (match(TK_LBRACKET)) {
                Opnd so = parse_assign_expr();
                if (bad()) return false;
                int64_t d;
                if (!const_dim_of(so, d)) return false;
                int64_t r;
                if (mul_ovf_(count, d, r)) { unsup(); return false; }
                count = r;
                if (!expect(TK_RBRACKET)) return false;
            }
            if (match(TK_COLON)) {  // bit-field width: parsed and ignored
                parse_assign_expr();
                if (bad()) return false;
            }
            if (count > 1) {
                if (count > 65536) { unsup(); return false; }
                for (int64_t q = 0; q < count; ++q)
                    fields.push(ar, SField{cat(ar, fname, S("_"), utoa(ar, (uint64_t)q)), fty});
                bool dup = false;
                for (uint32_t q = 0; q < farrs.n; ++q)
                    if (farrs[q].group == group && eq(farrs[q].base, fname)) {
                        farrs[q].count = (uint32_t)count;
                        dup = true;
                    }
                if (!dup) farrs.push(ar, FieldArr{name, fname, (uint32_t)count, group});
                any_arr = true;
            } else {
                fields.push(ar, SField{fname, fty});
            }
            if (!match(TK_COMMA)) break;
        }
        if (!expect(TK_SEMI)) return false;
    }
    if (!expect(TK_RBRACE)) return false;
    (void)any_arr;
    out = m.add_struct(name, fields.p, fields.n);
    snames.push(ar, StructName{name, out});
    if (at(TK_SEMI)) advance();
    return !bad();
}

// _zero_init_decl_fields (parser.py:2526-2536): every field gets a value;
// scalar fields are zero-initialized, nested structs recurse.
OCB_HD inline void Parser::zero_init_fields(Str prefix, Ty st) {
    uint32_t nf = m.nfields(st);
    for (uint32_t i = 0; i < nf && !bad(); ++i) {
        SField f = m.field(st, i);
        Str key = cat(ar, prefix, S("_"), f.name);
        uint32_t fv = new_val(key, f.ty);
        vars.set(ar, key, ov(fv));
        if (is_scalar_ty(f.ty)) {
            Opnd z = m.czero(f.ty);
            emit_bin(fv, BO_ADD, z, z);
        } else if (ty_is_struct(f.ty)) {
            if (++nest > MAX_NEST) { unsup(); --nest; return; }
            zero_init_fields(key, f.ty);
            --nest;
        }
    }
}

// Loads every field of the struct at `base` into `<prefix>_<field>` values:
// _load_struct_fields of a declaration (parser.py:2571-2594; pointer fields
// skipped, nested sentinels made when missing) and _load_param_fields of an
// inlined call (:1808-1845, `ptr_fields`: pointer fields loaded too).
OCB_HD inline void Parser::load_struct_fields(Opnd base, Ty st, Str prefix, uint32_t abs_off,
                                              uint32_t as, bool ptr_fields, bool) {
    uint32_t nf = m.nfields(st);
    for (uint32_t i = 0; i < nf && !bad(); ++i) {
        SField f = m.field(st, i);
        uint32_t off = m.field_offset(st, i) + abs_off;
        Str key = cat(ar, prefix, S("_"), f.name);
        bool load = is_scalar_ty(f.ty) || (ptr_fields && is_ptr(f.ty));
        if (load) {
            bool ok = true;
            Ty fp = ty_ptr(f.ty, as, false, ok);
            if (!ok) { unsup(); return; }
            uint32_t fa = new_val("faddr", fp);
            emit_bin(fa, BO_ADD, base, m.cint(S_INT32, off));
            uint32_t lv = new_val(key, f.ty);
            emit_load(lv, ov(fa));
            vars.set(ar, key, ov(lv));
        } else if (ty_is_struct(f.ty)) {
            if (!vars.has(key)) {
                uint32_t sv = new_val(key, f.ty);
                vars.set(ar, key, ov(sv));
            }
            if (++nest > MAX_NEST) { unsup(); --nest; return; }
            load_struct_fields(base, f.ty, key, off, as, ptr_fields, true);
            --nest;
        }
    }
}

// Struct-to-struct assignment `name = rhs` (parser.py:642-668, :3322-3348):
// each scalar field of rhs is copied into `<name>_<field>` when that key
// exists, then the sentinel is renewed under `name` if it carries another
// name.
OCB_HD inline void Parser::copy_struct_fields(uint32_t rhs, Str un) {
    Ty rt = m.vals[rhs].ty;
    uint32_t nf = m.nfields(rt);
    for (uint32_t i = 0; i < nf && !bad(); ++i) {
        SField f = m.field(rt, i);
        if (!is_scalar_ty(f.ty)) continue;
        Opnd src = struct_field_src(rhs, f.name);
        Str dk = cat(ar, un, S("_"), f.name);
        if (src.k != O_NONE && vars.has(dk)) {
            uint32_t nv = new_val(dk, f.ty);
            emit_bin(nv, BO_ADD, src, m.czero(f.ty));
            vars.set(ar, dk, ov(nv));
        }
    }
    Opnd *cs = vars.get(un);
    if (cs && isstruct(*cs) && !eq(vname(*cs), un)) {
        uint32_t fresh = new_val(un, tyof(*cs));
        vars.set(ar, un, ov(fresh));
    }
}

// `p.member` / `p->member` where p points to a struct (parser.py:1433-1527):
// the field's address, then its value (a nested struct stays an address).
OCB_HD inline Opnd Parser::member_of_ptr(Opnd lhs, Str member) {
    Ty st = ty_pointee(tyof(lhs));
    uint32_t as = ty_as(tyof(lhs));
    uint32_t n = field_array(st, member);
    if (n && at(TK_LBRACKET)) {
        advance();
        Opnd idx = parse_expr();
        if (bad() || !expect(TK_RBRACKET)) return lhs;
        int32_t f0 = field_or_raise(st, cat(ar, member, S("_0")));
        if (f0 < 0) return lhs;
        Ty et = m.field(st, (uint32_t)f0).ty;
        bool ok = true;
        Ty ep = ty_ptr(et, as, false, ok);
        if (!ok) { unsup(); return lhs; }
        uint32_t addr = new_val("faddr", ep);
        if (iscon(idx)) {
            int64_t k;
            if (!const_mod(idx, n, k)) return lhs;
            int32_t fk = field_or_raise(st, cat(ar, member, S("_"), utoa(ar, (uint64_t)k)));
            if (fk < 0) return lhs;
            emit_bin(addr, BO_ADD, lhs, m.cint(S_INT32, m.field_offset(st, (uint32_t)fk)));
        } else {
            uint32_t base = new_val("base", ep);
            emit_bin(base, BO_ADD, lhs, m.cint(S_INT32, m.field_offset(st, (uint32_t)f0)));
            Ty it = isval(idx) ? tyof(idx) : (Ty)S_INT32;
            uint32_t sc = new_val("scale", it);
            emit_bin(sc, BO_MUL, idx, m.cint(it, m.tsize(et)));
            emit_bin(addr, BO_ADD, ov(base), ov(sc));
        }
        if (ty_is_struct(et)) return ov(addr);
        uint32_t d = new_val(member, et);
        emit_load(d, ov(addr));
        return ov(d);
    }
    int32_t fi = field_or_raise(st, member);
    if (fi < 0) return lhs;
    Ty ft = m.field(st, (uint32_t)fi).ty;
    bool ok = true;
    Ty fp = ty_ptr(ft, as, false, ok);
    if (!ok) { unsup(); return lhs; }
    uint32_t addr = new_val("faddr", fp);
    emit_bin(addr, BO_ADD, lhs, m.cint(S_INT32, m.field_offset(st, (uint32_t)fi)));
    if (ty_is_struct(ft)) return ov(addr);
    uint32_t d = new_val(member, ft);
    emit_load(d, ov(addr));
    return ov(d);
}

// `s.member` of a struct variable (parser.py:1388-1431): the field's value in
// the variable map, made on first use; `src_name` receives the key.
OCB_HD inline Opnd Parser::member_of_struct(Opnd lhs, Str member, Str &src_name) {
    Ty st = tyof(lhs);
    Str vn = vname(lhs);
    uint32_t n = field_array(st, member);
    if (n && at(TK_LBRACKET)) {
        advance();
        Opnd idx = parse_expr();
        if (bad() || !expect(TK_RBRACKET)) return lhs;
        int32_t f0 = field_or_raise(st, cat(ar, member, S("_0")));
        if (f0 < 0) return lhs;
        Ty et = m.field(st, (uint32_t)f0).ty;
        int64_t k = 0;
        if (iscon(idx) && !const_mod(idx, n, k)) return lhs;
        Str key = cat(ar, vn, S("_"), cat(ar, member, S("_"), utoa(ar, (uint64_t)k)));
        if (!vars.has(key)) {
            uint32_t fv = new_val(key, et);
            vars.set(ar, key, ov(fv));
        }
        src_name = key;
        return *vars.get(key);
    }
    int32_t fi = field_or_raise(st, member);
    if (fi < 0) return lhs;
    Ty ft = m.field(st, (uint32_t)fi).ty;
    Str key = cat(ar, vn, S("_"), member);
    Opnd *o = vars.get(key);
    Opnd r;
    if (o) {
        r = *o;
    } else {
        uint32_t d = new_val(key, ft);
        vars.set(ar, key, ov(d));
        r = ov(d);
    }
    src_name = key;
    return r;
}

// The address of field `member` of the struct `addr` points to (the
// `faddr` steps of parser.py:3549-3567, :3645-3658).
OCB_HD inline Opnd Parser::field_addr(Opnd addr, Str member) {
    Ty st = ty_pointee(tyof(addr));
    int32_t fi = field_or_raise(st, member);
    if (fi < 0) return addr;
    bool ok = true;
    Ty fp = ty_ptr(m.field(st, (uint32_t)fi).ty, ty_as(tyof(addr)), false, ok);
    if (!ok) { unsup(); return addr; }
    uint32_t na = new_val("faddr", fp);
    emit_bin(na, BO_ADD, addr, m.cint(S_INT32, m.field_offset(st, (uint32_t)fi)));
    return ov(na);
}

// `.field` chains after a module variable's address (parser.py:3496-3522):
// while the current type is a struct, step to the field's address in the
// symbol's address space.
OCB_HD inline Opnd Parser::field_chain(Opnd addr, Ty cur_ty, uint32_t as) {
    while (!bad() && at(TK_DOT) && ty_is_struct(cur_ty)) {
        advance();
        if (!at(TK_IDENT)) { perr(); return addr; }
        Str f = peekv();
        advance();
        int32_t fi = field_or_raise(cur_ty, f);
        if (fi < 0) return addr;
        Ty ft = m.field(cur_ty, (uint32_t)fi).ty;
        bool ok = true;
        Ty fp = ty_ptr(ft, as, false, ok);
        if (!ok) { unsup(); return addr; }
        uint32_t na = new_val("faddr", fp);
        emit_bin(na, BO_ADD, addr, m.cint(S_INT32, m.field_offset(cur_ty, (uint32_t)fi)));
        addr = ov(na);
        cur_ty = ft;
    }
    return addr;
}

// `p->field = ...` / `p.field = ...` of a pointer to a struct
// (parser.py:3526-3591): the field's address, through array members,
// nested fields and a pointer field's element.
OCB_HD inline Opnd Parser::member_lvalue(Opnd var) {
    advance();  // '->' or '.'
    if (!at(TK_IDENT)) { perr(); return onone(); }
    Str member = peekv();
    advance();
    Ty st = ty_pointee(tyof(var));
    uint32_t as = ty_as(tyof(var));
    Opnd addr;
    uint32_t n = field_array(st, member);
    if (n && at(TK_LBRACKET)) {
        advance();
        Opnd idx = parse_expr();
        if (bad() || !expect(TK_RBRACKET)) return onone();
        int32_t f0 = field_or_raise(st, cat(ar, member, S("_0")));
        if (f0 < 0) return onone();
        Ty ft = m.field(st, (uint32_t)f0).ty;
        bool ok = true;
        Ty fp = ty_ptr(ft, as, false, ok);
        if (!ok) { unsup(); return onone(); }
        uint32_t ba = new_val("faddr", fp);
        emit_bin(ba, BO_ADD, var, m.cint(S_INT32, m.field_offset(st, (uint32_t)f0)));
        uint32_t es = m.tsize(ft);
        if (es != 1) {
            Ty it = isval(idx) ? tyof(idx) : (Ty)S_INT32;
            uint32_t sc = new_val("scale", it);
            emit_bin(sc, BO_MUL, idx, m.cint(it, es));
            idx = ov(sc);
        }
        uint32_t a = new_val("faddr", fp);
        emit_bin(a, BO_ADD, ov(ba), idx);
        addr = ov(a);
    } else {
        addr = field_addr(var, member);
    }
    while (!bad() && (at(TK_DOT) || at(TK_ARROW))) {
        advance();
        if (!at(TK_IDENT)) { perr(); return onone(); }
        Str sub = peekv();
        advance();
        if (!isptr_struct(addr)) break;
        addr = field_addr(addr, sub);
    }
    if (bad()) return onone();
    Ty at_ = tyof(addr);
    if (at(TK_LBRACKET) && is_ptr(at_) && is_ptr(ty_pointee(at_))) {  // p->ptr_field[i]
        Ty pf = ty_pointee(at_);
        uint32_t pv = new_val("pfield", pf);
        emit_load(pv, addr);
        advance();
        Opnd idx = parse_expr();
        if (bad() || !expect(TK_RBRACKET)) return onone();
        Ty et = ty_pointee(pf);
        uint32_t es = m.tsize(et);
        if (es != 1) {
            Ty it = isval(idx) ? tyof(idx) : (Ty)S_INT32;
            uint32_t sc = new_val("scale", it);
            emit_bin(sc, BO_MUL, idx, m.cint(it, es));
            idx = ov(sc);
        }
        bool ok = true;
        Ty ep = ty_ptr(et, ty_as(pf), false, ok);
        if (!ok) { unsup(); return onone(); }
        uint32_t ea = new_val("addr", ep);
        emit_bin(ea, BO_ADD, ov(pv), idx);
        addr = ov(ea);
    }
    return addr;
}

// _parse_compound_literal (parser.py:2251-2283): `(T){v0, v1, ...}`
OCB_HD inline Opnd Parser::parse_compound_literal(Ty st) {
    if (!expect(TK_LBRACE)) return onone();
    Vec<Opnd> vals;
    vals.init();
    if (!at(TK_RBRACE)) {
        vals.push(ar, parse_assign_expr());
        while (!bad() && match(TK_COMMA)) {
            if (at(TK_RBRACE)) break;
            vals.push(ar, parse_assign_expr());
        }
    }
    if (bad() || !expect(TK_RBRACE)) return onone();
    uint32_t d = new_val("compound", st);
    if (bad()) return onone();
    uint32_t did = m.vals[d].id;
    uint32_t nf = m.nfields(st);
    // dict of this id, filled in field order (zip stops at the shorter list)
    for (uint32_t i = 0; i < nf && i < vals.n && !bad(); ++i) {
        SField f = m.field(st, i);
        if (!is_scalar_ty(f.ty)) continue;
        Str key = cat(ar, m.vals[d].name, S("_"), f.name);
        uint32_t fv = new_val(key, f.ty);
        emit_bin(fv, BO_ADD, vals[i], m.czero(f.ty));
        isrf_set(did, f.name, ov(fv));
        vars.set(ar, key, ov(fv));
    }
    return ov(d);
}

// _flat_struct_params (parser.py:3812-3835): one ParamInst per leaf field,
// named `<prefix>_<field>`; names already bound are skipped.
OCB_HD inline void Parser::flat_struct_params(Str prefix, Ty st, uint32_t slot, NameSet &seen,
                                              uint32_t &next) {
    uint32_t nf = m.nfields(st);
    for (uint32_t i = 0; i < nf && !bad(); ++i) {
        SField f = m.field(st, i);
        Str key = cat(ar, prefix, S("_"), f.name);
        if (seen.has(key)) continue;
        if (ty_is_struct(f.ty)) {
            uint32_t sv = new_val(key, f.ty);
            vars.set(ar, key, ov(sv));
            seen.add(ar, key);
            if (++nest > MAX_NEST) { unsup(); --nest; return; }
            flat_struct_params(key, f.ty, slot, seen, slot);
            --nest;
        } else {
            uint32_t pv = new_val(key, f.ty);
            Inst pi = mk_inst(I_PARAM, 0, (int32_t)pv, onone(), onone());
            pi.pidx = slot;
            pi.func = key;
            emit(pi);
            vars.set(ar, key, ov(pv));
            seen.add(ar, key);
            slot++;
        }
    }
    next = slot;
}

}  // namespace cc
}  // namespace ocb
