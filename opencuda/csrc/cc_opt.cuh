// IR optimizer: restates opencuda/ir/optimize.py (passes and the pass
// schedule of optimize(), :1443-1607) and opencuda/ir/unroll.py for one
// kernel at a time, on the IR built by the parser.  Every pass keeps the
// reference's visiting order, its in-place mutation of instructions and its
// change counts (the counts steer the fixpoint loops of the schedule).
//
// Constants carry Python semantics: an int (pyint) or a float, whatever the
// IR type says; folds follow Python's int/float arithmetic.
#pragma once
#include "cc_opt_base.cuh"

namespace ocb {
namespace cc {

// ---------------------------------------------------------------------------
// the optimizer of one kernel
// ---------------------------------------------------------------------------
struct Opt {
    Module &m;
    Arena &ar;   // the IR's arena (persistent)
    Arena &tmp;  // per-pass scratch, reset between passes
    Kernel *k;

    OCB_HD Opt(Module &mod, Arena &tmp_) : m(mod), ar(*mod.ar), tmp(tmp_), k(nullptr) {}

    // m.raises: a Python exception the reference raises inside optimize()
    OCB_HD bool bad() const { return m.unsup || m.raises || ar.oom || tmp.oom; }
#ifdef OCB_TRAP_UNSUP
    void unsup(int line = __builtin_LINE()) {
        fprintf(stderr, "opt unsupported at cc_opt.cuh:%d\n", line);
        m.unsup = true;
    }
#else
    OCB_HD void unsup() { m.unsup = true; }
#endif
    OCB_HD Inst &I(uint32_t ix) { return m.insts[ix]; }
    OCB_HD Block &B(uint32_t b) { return m.blocks[b]; }
    OCB_HD uint32_t vid(Opnd o) const { return m.vals[o.x].id; }
    OCB_HD uint32_t did(const Inst &i) const { return m.vals[(uint32_t)i.dest].id; }
    OCB_HD bool has_dest(const Inst &i) const { return i.dest >= 0; }
    OCB_HD Ty dty(const Inst &i) const { return m.vals[(uint32_t)i.dest].ty; }
    OCB_HD PyVal cv(Opnd o) const { return pv_of(m.consts[o.x]); }
    OCB_HD bool cis(Opnd o, pyint v) const { return o.k == O_CONST && pv_eq_int(cv(o), v); }
    OCB_HD uint32_t new_value(const char *name, Ty ty) {
        return m.add_val(k->next_id++, ty, S(name));
    }
    OCB_HD uint32_t new_value(Str name, Ty ty) { return m.add_val(k->next_id++, ty, name); }
    OCB_HD Opnd cint(Ty t, pyint v) { return m.cint(t, v); }
    OCB_HD Opnd cflt(Ty t, double v) { return m.cfloat(t, v); }
    OCB_HD Opnd cpv(Ty t, const PyVal &v) { return v.isf ? m.cfloat(t, v.f) : m.cint(t, v.i); }
    OCB_HD uint32_t add_inst(const Inst &i) { return m.add_inst(i); }
    OCB_HD uint32_t nid() const { return k->next_id; }
    OCB_HD void reset_tmp() {
        tmp.used = 0;
    }
    // dest ids of all instructions (hasattr(inst,'dest') and inst.dest is not None)
    OCB_HD IdArr<uint32_t> def_counts() {
        IdArr<uint32_t> dc;
        dc.init(tmp, nid(), 0);
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (in.dest >= 0) {
                    uint32_t d = did(in);
                    dc.set(d, dc.get(d) + 1);
                }
            }
        }
        return dc;
    }
    OCB_HD void set_br(uint32_t b, Str t) { B(b).term = Term{T_BR, onone(), t, Str{nullptr, 0}}; }

    // ---- _fold_bin (optimize.py:73-106) -----------------------------------
    // Result: 0 = None, 1 = value in *out (exact), 2 = int value known only
    // modulo 2^128 (the caller masks it, or declines the TU)
    OCB_HD int fold_bin(uint8_t op, PyVal a, PyVal b, bool is_float, PyVal &out) {
        if (is_float) {
            double x = pv_to_float(a), y = pv_to_float(b);
            switch (op) {
            case BO_ADD: out = pv_float(x + y); return 1;
            case BO_SUB: out = pv_float(x - y); return 1;
            case BO_MUL: out = pv_float(x * y); return 1;
            case BO_DIV:
                if (y != 0.0) { out = pv_float(x / y); return 1; }
                return 0;
            case BO_MOD:
                if (y != 0.0) { out = pv_float(py_fmod(x, y)); return 1; }
                return 0;
            default: break;
            }
            PyVal ia, ib;
            pyint xi, yi;
            if (!pv_to_int(pv_float(x), xi) || !pv_to_int(pv_float(y), yi)) {
                if (!is_finite(x) || !is_finite(y)) return 0;  // int() raises: no fold
                unsup();
                return 0;
            }
            ia = pv_int(xi);
            ib = pv_int(yi);
            return fold_int(op, ia.i, ib.i, out);
        }
        pyint x, y;
        if (!pv_to_int(a, x) || !pv_to_int(b, y)) {
            bool fa = a.isf && !is_finite(a.f), fb = b.isf && !is_finite(b.f);
            if (fa || fb) return 0;  // int(nan/inf) raises inside the try: None
            unsup();
            return 0;
        }
        return fold_int(op, x, y, out);
    }
    OCB_HD int fold_int(uint8_t op, pyint x, pyint y, PyVal &out) {
        switch (op) {
        case BO_ADD: out = pv_int(x + y); return py_ok(out.i) ? 1 : 2;
        case BO_SUB: out = pv_int(x - y); return py_ok(out.i) ? 1 : 2;
        case BO_MUL: {
            pyint r;
            if (py_mul(x, y, r)) { out = pv_int(r); return 1; }
            out = pv_int((pyint)((unsigned __int128)x * (unsigned __int128)y));
            return 2;
        }
        case BO_DIV: {
            if (y == 0) return 0;
            pyint q = py_abs(x) / py_abs(y);
            out = pv_int(((x >= 0) == (y >= 0)) ? q : -q);
            return 1;
        }
        case BO_MOD: {
            if (y == 0) return 0;
            pyint q = py_abs(x) / py_abs(y);
            pyint rem = py_abs(x) - q * py_abs(y);
            out = pv_int(x >= 0 ? rem : -rem);
            return 1;
        }
        case BO_AND: out = pv_int(x & y); return 1;
        case BO_OR: out = pv_int(x | y); return 1;
        case BO_XOR: out = pv_int(x ^ y); return 1;
        case BO_SHL: {
            if (y < 0) return 0;  // ValueError: negative shift count
            pyint r;
            if (py_shl(x, y, r)) { out = pv_int(r); return 1; }
            out = pv_int(y >= 128 ? 0 : (pyint)((unsigned __int128)x << (int)y));
            return 2;
        }
        case BO_SHR:
            if (y < 0) return 0;
            out = pv_int(py_shr(x, y));
            return 1;
        }
        return 0;
    }

    // ---- constant_fold (optimize.py:109-387) -------------------------------
    OCB_HD uint32_t constant_fold() {
        uint32_t folded = 0;
        // per-block replacements: id -> const operand; stamp = block ordinal
        uint32_t n0 = nid();
        IdArr<uint32_t> stamp;
        stamp.init(tmp, n0, 0xFFFFFFFFu);
        Opnd *rep = (Opnd *)tmp.alloc(sizeof(Opnd) * (uint64_t)(n0 ? n0 : 1), 16);
        if (!rep || bad()) return 0;
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            uint32_t bidx = k->blocks[bi];
            auto resolve = [&](Opnd o) -> Opnd {
                if (o.k == O_VAL) {
                    uint32_t id = vid(o);
                    if (stamp.get(id) == bi) return rep[id];  // always a Const
                }
                return o;
            };
            Vec<uint32_t> nl;
            nl.init();
            bool rebuilt = false;
            Vec<uint32_t> &old = B(bidx).insts;
            for (uint32_t ii = 0; ii < old.n; ++ii) {
                uint32_t ix = old[ii];
                Inst &in = I(ix);
                if (in.kind == I_BIN) {
                    in.a = resolve(in.a);
                    in.b = resolve(in.b);
                    Ty dt = dty(in);
                    bool is_float = ty_is_float(dt);
                    bool lc = in.a.k == O_CONST, rc = in.b.k == O_CONST;
                    PyVal lv = lc ? cv(in.a) : PyVal{}, rv = rc ? cv(in.b) : PyVal{};
                    PyVal res;
                    int fr = (lc && rc) ? fold_bin(in.op, lv, rv, is_float, res) : 0;
                    if (bad()) return folded;
                    bool rv_int = rc && !rv.isf, lv_int = lc && !lv.isf;
                    auto pow2 = [](pyint v) { return v > 0 && (v & (v - 1)) == 0; };
                    if (fr) {
                        Opnd fc;
                        if (is_float) {
                            if (fr == 2) { unsup(); return folded; }
                            fc = cpv(dt, res);
                            in.a = fc;
                            in.b = cflt(dt, 0.0);
                        } else {
                            if (!masks(dt) && fr == 2) { unsup(); return folded; }
                            pyint v = res.i;
                            if (masks(dt)) {
                                if (ty_size(dt) == 0) { unsup(); return folded; }
                                v = mask_int_wrapped(res.i, dt);
                            }
                            fc = cint(dt, v);
                            in.a = fc;
                            in.b = cint(dt, 0);
                        }
                        in.op = BO_ADD;
                        uint32_t id = did(in);
                        if (stamp.set(id, bi)) rep[id] = fc;
                        else { unsup(); return folded; }
                        folded++;
                    } else if (in.op == BO_MUL && rc && pv_eq_int(rv, 1) && in.a.k == O_VAL) {
                        in.op = BO_ADD;
                        in.b = is_float ? cflt(dt, 0.0) : cint(dt, 0);
                        folded++;
                    } else if (in.op == BO_MUL && lc && pv_eq_int(lv, 1) && in.b.k == O_VAL) {
                        in.op = BO_ADD;
                        in.a = in.b;
                        in.b = is_float ? cflt(dt, 0.0) : cint(dt, 0);
                        folded++;
                    } else if (in.op == BO_DIV && rc && pv_eq_int(rv, 1) && in.a.k == O_VAL) {
                        in.op = BO_ADD;
                        in.b = cint(dt, 0);
                        folded++;
                    } else if (!is_float && in.op == BO_MUL && rv_int && pow2(rv.i)) {
                        in.op = BO_SHL;
                        in.b = cint(dt, py_bitlen(rv.i) - 1);
                        folded++;
                    } else if (!is_float && in.op == BO_MUL && lv_int && pow2(lv.i)) {
                        in.op = BO_SHL;
                        in.a = in.b;
                        in.b = cint(dt, py_bitlen(lv.i) - 1);
                        folded++;
                    } else if (!is_float && in.op == BO_DIV && rv_int && rv.i > 1 && pow2(rv.i) &&
                               !is_ptr(dt) && !ty_is_signed(dt)) {
                        in.op = BO_SHR;
                        in.b = cint(dt, py_bitlen(rv.i) - 1);
                        folded++;
                    } else if (!is_float && in.op == BO_DIV && rv_int && rv.i > 1 && pow2(rv.i) &&
                               !is_ptr(dt) && ty_is_signed(dt)) {
                        int kk = py_bitlen(rv.i) - 1;
                        int bits = (int)ty_size(dt) * 8;
                        Ty tu = bits == 32 ? S_UINT32 : S_UINT64;
                        Opnd n = in.a;
                        uint32_t t1 = new_value("_sdiv_sign", dt);
                        uint32_t t2 = new_value("_sdiv_bias", tu);
                        uint32_t t3 = new_value("_sdiv_adj", dt);
                        if (!rebuilt) { nl = old.copy(ar); nl.n = ii; rebuilt = true; }
                        nl.push(ar, add_inst(mk_inst(I_BIN, BO_SHR, (int32_t)t1, n, cint(dt, bits - 1))));
                        nl.push(ar, add_inst(mk_inst(I_BIN, BO_SHR, (int32_t)t2, ov(t1), cint(tu, bits - kk))));
                        nl.push(ar, add_inst(mk_inst(I_BIN, BO_ADD, (int32_t)t3, n, ov(t2))));
                        Inst &in2 = I(ix);  // m.insts may have grown
                        in2.op = BO_SHR;
                        in2.a = ov(t3);
                        in2.b = cint(dt, kk);
                        folded++;
                    } else if (!is_float && in.op == BO_MOD && rv_int && pow2(rv.i) && !is_ptr(dt) &&
                               !ty_is_signed(dt)) {
                        in.op = BO_AND;
                        in.b = cint(dt, rv.i - 1);
                        folded++;
                    } else if (!is_float && in.op == BO_MOD && rv_int && pow2(rv.i) && !is_ptr(dt) &&
                               ty_is_signed(dt)) {
                        int kk = py_bitlen(rv.i) - 1;
                        int bits = (int)ty_size(dt) * 8;
                        Ty tu = bits == 32 ? S_UINT32 : S_UINT64;
                        Opnd n = in.a;
                        uint32_t t1 = new_value("_smod_sign", dt);
                        uint32_t t2 = new_value("_smod_bias", tu);
                        uint32_t t3 = new_value("_smod_adj", dt);
                        uint32_t t4 = new_value("_smod_masked", dt);
                        if (!rebuilt) { nl = old.copy(ar); nl.n = ii; rebuilt = true; }
                        nl.push(ar, add_inst(mk_inst(I_BIN, BO_SHR, (int32_t)t1, n, cint(dt, bits - 1))));
                        nl.push(ar, add_inst(mk_inst(I_BIN, BO_SHR, (int32_t)t2, ov(t1), cint(tu, bits - kk))));
                        nl.push(ar, add_inst(mk_inst(I_BIN, BO_ADD, (int32_t)t3, n, ov(t2))));
                        nl.push(ar, add_inst(mk_inst(I_BIN, BO_AND, (int32_t)t4, ov(t3), cint(dt, rv.i - 1))));
                        Inst &in2 = I(ix);
                        in2.op = BO_SUB;
                        in2.a = ov(t4);
                        in2.b = ov(t2);
                        folded++;
                    } else if (in.op == BO_MUL && ((rc && pv_eq_int(rv, 0)) || (lc && pv_eq_int(lv, 0)))) {
                        in.a = cint(dt, 0);
                        in.b = cint(dt, 0);
                        in.op = BO_ADD;
                        folded++;
                    } else if (!is_float && in.op == BO_AND &&
                               ((rc && pv_eq_int(rv, 0)) || (lc && pv_eq_int(lv, 0)))) {
                        in.a = cint(dt, 0);
                        in.b = cint(dt, 0);
                        in.op = BO_ADD;
                        folded++;
                    } else if (!is_float && in.op == BO_AND && !is_ptr(dt)) {
                        if (ty_size(dt) == 0) { unsup(); return folded; }
                        pyint ones = mask_int_wrapped(-1, dt);
                        if (rc && pv_eq_int(rv, ones) && in.a.k == O_VAL) {
                            in.op = BO_ADD;
                            in.b = cint(dt, 0);
                            folded++;
                        } else if (lc && pv_eq_int(lv, ones) && in.b.k == O_VAL) {
                            in.op = BO_ADD;
                            in.a = in.b;
                            in.b = cint(dt, 0);
                            folded++;
                        }
                    } else if (!is_float && in.op == BO_OR && !is_ptr(dt)) {
                        if (ty_size(dt) == 0) { unsup(); return folded; }
                        pyint ones = mask_int_wrapped(-1, dt);
                        if ((rc && pv_eq_int(rv, ones)) || (lc && pv_eq_int(lv, ones))) {
                            in.a = cint(dt, ones);
                            in.b = cint(dt, 0);
                            in.op = BO_ADD;
                            folded++;
                        }
                    } else if (!is_float && (in.op == BO_SUB || in.op == BO_XOR) && in.a.k == O_VAL &&
                               in.b.k == O_VAL && vid(in.a) == vid(in.b)) {
                        in.a = cint(dt, 0);
                        in.b = cint(dt, 0);
                        in.op = BO_ADD;
                        folded++;
                    } else if (!is_float && (in.op == BO_AND || in.op == BO_OR) && in.a.k == O_VAL &&
                               in.b.k == O_VAL && vid(in.a) == vid(in.b)) {
                        in.op = BO_ADD;
                        in.b = cint(dt, 0);
                        folded++;
                    }
                } else if (in.kind == I_CMP) {
                    in.a = resolve(in.a);
                    in.b = resolve(in.b);
                } else if (in.kind == I_CVT) {
                    Opnd src = resolve(in.a);
                    in.a = src;
                    if (src.k == O_CONST) {
                        Ty dt = dty(in);
                        bool dfl = ty_is_float(dt);
                        const Const &sc = m.consts[src.x];
                        bool sfl = ty_is_float(sc.ty);
                        PyVal sv = pv_of(sc);
                        bool ok = true;
                        PyVal fv;
                        if (dfl) {
                            fv = pv_float(pv_to_float(sv));
                        } else {
                            PyVal raw = sfl ? pv_float(pv_to_float(sv)) : sv;
                            pyint iv;
                            if (!pv_to_int(raw, iv)) {
                                if (raw.isf && !is_finite(raw.f)) ok = false;  // raises: kept
                                else { unsup(); return folded; }
                            } else {
                                if (masks(dt)) {
                                    if (ty_size(dt) == 0) { unsup(); return folded; }
                                    iv = mask_int_wrapped(iv, dt);
                                }
                                fv = pv_int(iv);
                            }
                        }
                        if (ok) {
                            Opnd l = cpv(dt, fv);
                            Opnd r = dfl ? cflt(dt, 0.0) : cint(dt, 0);
                            uint32_t nb = add_inst(mk_inst(I_BIN, BO_ADD, I(ix).dest, l, r));
                            if (!rebuilt) { nl = old.copy(ar); nl.n = ii; rebuilt = true; }
                            nl.push(ar, nb);
                            folded++;
                            continue;
                        }
                    }
                } else if (in.kind == I_LOAD) {
                    in.a = resolve(in.a);
                } else if (in.kind == I_STORE) {
                    in.a = resolve(in.a);
                    in.b = resolve(in.b);
                }
                if (rebuilt) nl.push(ar, ix);
            }
            if (rebuilt) B(bidx).insts = nl;
            Term &t = B(bidx).term;
            if (t.kind == T_CBR) {
                Opnd c = t.v.k == O_VAL ? resolve(t.v) : t.v;
                if (c.k == O_CONST) {
                    Str tg = pv_truthy(cv(c)) ? t.t : t.f;
                    set_br(bidx, tg);
                    folded++;
                }
            }
            if (bad()) return folded;
        }
        return folded;
    }

    // ---- cse (optimize.py:397-640) -------------------------------------------
    OCB_HD uint32_t cse() {
        IdArr<uint32_t> gdc = def_counts();
        uint32_t n0 = nid();
        uint32_t eliminated = 0;
        // global replacements: id -> value index (0xFFFFFFFF none)
        IdArr<uint32_t> grep;
        grep.init(tmp, n0, 0xFFFFFFFFu);
        // predecessor lists (with duplicates, like the reference's list)
        LabelMap lm;
        lm.build(tmp, m, k->blocks);
        uint32_t nb = k->blocks.n;
        uint32_t *npred = (uint32_t *)tmp.alloc(4ull * (nb + 1), 16);
        int32_t *pred0 = (int32_t *)tmp.alloc(4ull * (nb + 1), 16);
        Seen *final_seen = (Seen *)tmp.alloc(sizeof(Seen) * (uint64_t)(nb + 1), 16);
        uint8_t *has_final = (uint8_t *)tmp.alloc(nb + 1, 16);
        // block ordinal by label (the reference keys dicts by label: last wins)
        if (!npred || !pred0 || !final_seen || !has_final || bad()) return 0;
        IdArr<uint32_t> ord_of_block;  // block index -> ordinal
        ord_of_block.init(tmp, m.blocks.n, 0xFFFFFFFFu);
        for (uint32_t i = 0; i < nb; ++i) {
            npred[i] = 0;
            pred0[i] = -1;
            has_final[i] = 0;
        }
        // the dict {bb.label: []} has one entry per distinct label: use the
        // ordinal of the last block with that label
        for (uint32_t i = 0; i < nb; ++i) ord_of_block.set(k->blocks[i], i);
        auto lab_ord = [&](Str l) -> int32_t {
            int32_t b = lm.get(l);
            return b < 0 ? -1 : (int32_t)ord_of_block.get((uint32_t)b);
        };
        for (uint32_t i = 0; i < nb; ++i) {
            Block &b = B(k->blocks[i]);
            const Term &t = b.term;
            Str tg[2];
            int nt = 0;
            if (t.kind == T_BR) tg[nt++] = t.t;
            else if (t.kind == T_CBR) { tg[nt++] = t.t; tg[nt++] = t.f; }
            for (int q = 0; q < nt; ++q) {
                int32_t o = lab_ord(tg[q]);
                if (o < 0) continue;
                if (npred[o] == 0) pred0[o] = (int32_t)i;
                npred[o]++;
            }
        }
        // With unique labels a block's final table is read only by the later
        // blocks whose single predecessor it is; the last of them takes the
        // table itself instead of a copy (nothing reads it afterwards).
        uint32_t *readers = nullptr;
        {
            size_t mark = tmp.used;
            LabelSet ls;
            ls.init(tmp, nb + 2);
            bool uniq = ls.cap != 0;
            for (uint32_t i = 0; i < nb && uniq; ++i) uniq = ls.add(B(k->blocks[i]).label);
            tmp.used = mark;
            if (uniq) {
                readers = (uint32_t *)tmp.alloc(4ull * (nb + 1), 16);
                if (!readers) return 0;
                for (uint32_t i = 0; i < nb; ++i) readers[i] = 0;
                for (uint32_t i = 0; i < nb; ++i)
                    if (npred[i] == 1 && pred0[i] >= 0 && (uint32_t)pred0[i] < i) readers[pred0[i]]++;
            }
        }
        IdArr<uint32_t> rstamp;  // per-block replacements: stamp = ordinal
        rstamp.init(tmp, n0, 0xFFFFFFFFu);
        uint32_t *rval = (uint32_t *)tmp.alloc(4ull * (n0 ? n0 : 1), 16);
        IdArr<uint32_t> wstamp;  // written_ids
        wstamp.init(tmp, n0, 0xFFFFFFFFu);
        if (!rval || bad()) return 0;
        bool any_rep = false;
        for (uint32_t bi = 0; bi < nb; ++bi) {
            uint32_t bidx = k->blocks[bi];
            Block &b = B(bidx);
            int32_t my = lab_ord(b.label);
            Seen seen;
            // pred lists are keyed by label; a duplicate label shares the last one's
            uint32_t np = my >= 0 ? npred[my] : 0;
            int32_t p0 = my >= 0 ? pred0[my] : -1;
            if (np == 1 && p0 >= 0 && has_final[lab_ord(B(k->blocks[p0]).label)]) {
                int32_t po = lab_ord(B(k->blocks[p0]).label);
                if (readers && --readers[po] == 0) seen = final_seen[po];
                else if (!seen.copy_from(tmp, final_seen[po])) return eliminated;
            } else {
                if (!seen.init(tmp, 64, m.consts.p)) return eliminated;
            }
            auto in_rep = [&](uint32_t id) { return rstamp.get(id) == bi; };
            auto rep1 = [&](Opnd o) -> Opnd {  // single-step replacement
                if (o.k == O_VAL && in_rep(vid(o))) return ov(rval[vid(o)]);
                return o;
            };
            auto key = [&](Opnd o) -> OKey {
                OKey r;
                if (o.k == O_VAL) {
                    uint32_t v = o.x;
                    uint32_t guard = 0;
                    while (in_rep(m.vals[v].id)) {
                        v = rval[m.vals[v].id];
                        if (++guard > 1000000) { unsup(); break; }
                    }
                    r.tag = 1;
                    r.x = m.vals[v].id;
                    return r;
                }
                // A NaN constant: Python compares ('const', nan) keys by object
                // identity (equal only to itself); the constant index plays the
                // object's part (a propagated constant keeps its index, every
                // fold makes a new one), and okey_eq compares indices first.
                r.tag = 0;
                r.x = o.x;
                return r;
            };
            auto written = [&](uint32_t id) { return wstamp.get(id) == bi; };
            auto mark_written = [&](uint32_t id) {
                if (!wstamp.set(id, bi)) unsup();
            };
            Vec<uint32_t> rep_ids;
            rep_ids.init();
            auto add_rep = [&](uint32_t id, uint32_t v) {
                if (!rstamp.set(id, bi)) { unsup(); return; }
                rval[id] = v;
                rep_ids.push(tmp, id);
            };
            uint32_t w = 0;
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                uint32_t ix = b.insts[ii];
                Inst &in = I(ix);
                bool keep = true;
                if (in.kind == I_BIN) {
                    in.a = rep1(in.a);
                    in.b = rep1(in.b);
                    uint32_t d = did(in);
                    if (written(d)) {
                    } else if (gdc.get(d) >= 2) {
                        mark_written(d);
                    } else {
                        CKey ck;
                        ck.kind = 0;
                        ck.op = in.op;
                        OKey lk = key(in.a), rk = key(in.b);
                        bool comm = in.op == BO_ADD || in.op == BO_MUL || in.op == BO_AND ||
                                    in.op == BO_OR || in.op == BO_XOR;
                        if (comm && okey_gt(lk, rk, m.consts.p)) { OKey t = lk; lk = rk; rk = t; }
                        ck.l = lk;
                        ck.r = rk;
                        ck.t1 = ty_strkey(dty(in));
                        ck.t2 = 0;
                        int32_t f = seen.find(ck);
                        if (f >= 0) {
                            add_rep(d, (uint32_t)f);
                            eliminated++;
                            keep = false;
                        } else {
                            if (!seen.put(tmp, ck, (uint32_t)in.dest)) return eliminated;
                            mark_written(d);
                        }
                    }
                } else if (in.kind == I_CVT) {
                    in.a = rep1(in.a);
                    uint32_t d = did(in);
                    if (!written(d) && gdc.get(d) < 2) {
                        CKey ck;
                        ck.kind = 1;
                        ck.op = 0;
                        ck.l = key(in.a);
                        ck.r = OKey{0, 0};
                        ck.t1 = ty_strkey(dty(in));
                        ck.t2 = ty_strkey(m.opty(in.a));
                        int32_t f = seen.find(ck);
                        if (f >= 0) {
                            add_rep(d, (uint32_t)f);
                            eliminated++;
                            keep = false;
                        } else {
                            if (!seen.put(tmp, ck, (uint32_t)in.dest)) return eliminated;
                            mark_written(d);
                        }
                    }
                } else if (in.kind == I_CMP) {
                    in.a = rep1(in.a);
                    in.b = rep1(in.b);
                    uint32_t d = did(in);
                    if (!written(d) && gdc.get(d) < 2) {
                        OKey lk = key(in.a), rk = key(in.b);
                        uint8_t op = in.op;
                        if ((op == CO_EQ || op == CO_NE) && okey_gt(lk, rk, m.consts.p)) {
                            OKey t = lk; lk = rk; rk = t;
                        } else if ((op == CO_LT || op == CO_GT || op == CO_LE || op == CO_GE) &&
                                   okey_gt(lk, rk, m.consts.p)) {
                            OKey t = lk; lk = rk; rk = t;
                            op = op == CO_LT ? CO_GT : op == CO_GT ? CO_LT : op == CO_LE ? CO_GE : CO_LE;
                        }
                        CKey ck;
                        ck.kind = 2;
                        ck.op = op;
                        ck.l = lk;
                        ck.r = rk;
                        ck.t1 = ck.t2 = 0;
                        int32_t f = seen.find(ck);
                        if (f >= 0) {
                            add_rep(d, (uint32_t)f);
                            eliminated++;
                            keep = false;
                        } else {
                            if (!seen.put(tmp, ck, (uint32_t)in.dest)) return eliminated;
                            mark_written(d);
                        }
                    }
                } else if (in.kind == I_CALL) {
                    uint32_t pb = in.dest >= 0 ? pure_builtin_code(in.func) : 0;
                    if (pb) {
                        uint32_t d = did(in);
                        if (!written(d) && gdc.get(d) < 2) {
                            CKey ck;
                            ck.kind = 3;
                            ck.op = (uint8_t)pb;
                            ck.l = ck.r = OKey{0, 0};
                            ck.t1 = ck.t2 = 0;
                            int32_t f = seen.find(ck);
                            if (f >= 0) {
                                add_rep(d, (uint32_t)f);
                                eliminated++;
                                keep = false;
                            } else {
                                if (!seen.put(tmp, ck, (uint32_t)in.dest)) return eliminated;
                                mark_written(d);
                            }
                        }
                    }
                } else if (in.kind == I_LOAD) {
                    in.a = rep1(in.a);
                } else if (in.kind == I_STORE) {
                    in.a = rep1(in.a);
                    in.b = rep1(in.b);
                } else if (in.kind == I_PRINTF && in.args.n) {
                    Vec<Opnd> na = in.args.copy(ar);
                    for (uint32_t q = 0; q < na.n; ++q) na[q] = rep1(na[q]);
                    in.args = na;
                }
                if (bad()) return eliminated;
                if (keep) b.insts[w++] = ix;
            }
            b.insts.n = w;
            // global_replacements.update(replacements)
            for (uint32_t q = 0; q < rep_ids.n; ++q) {
                grep.set(rep_ids[q], rval[rep_ids[q]]);
                any_rep = true;
            }
            if (my >= 0) {
                final_seen[my] = seen;
                has_final[my] = 1;
            }
        }
        if (any_rep) {
            auto chase = [&](Opnd o) -> Opnd {
                if (o.k != O_VAL) return o;
                uint32_t v = o.x, guard = 0;
                while (grep.get(m.vals[v].id) != 0xFFFFFFFFu) {
                    v = grep.get(m.vals[v].id);
                    if (++guard > 1000000) { unsup(); break; }
                }
                return ov(v);
            };
            for (uint32_t bi = 0; bi < nb; ++bi) {
                Block &b = B(k->blocks[bi]);
                for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                    Inst &in = I(b.insts[ii]);
                    switch (in.kind) {
                    case I_BIN:
                    case I_CMP:
                    case I_STORE:
                        in.a = chase(in.a);
                        in.b = chase(in.b);
                        break;
                    case I_CVT:
                    case I_LOAD: in.a = chase(in.a); break;
                    case I_CALL:
                    case I_PRINTF:
                        if (in.args.n) {
                            Vec<Opnd> na = in.args.copy(ar);
                            for (uint32_t q = 0; q < na.n; ++q) na[q] = chase(na[q]);
                            in.args = na;
                        }
                        break;
                    default: break;
                    }
                }
                Term &t = b.term;
                if (t.kind == T_CBR && t.v.k == O_VAL) t.v = chase(t.v);
            }
        }
        return eliminated;
    }
    // 1..12 for the builtins CSE treats as pure (optimize.py:555-575:
    // thread/block index and dimension reads), 0 for any other call
    OCB_HD static uint32_t pure_builtin_code(Str f) {
        const char *names[12] = {"threadIdx.x", "threadIdx.y", "threadIdx.z",
                                 "blockIdx.x",  "blockIdx.y",  "blockIdx.z",
                                 "blockDim.x",  "blockDim.y",  "blockDim.z",
                                 "gridDim.x",   "gridDim.y",   "gridDim.z"};
        if (f.n < 9 || f.n > 11) return 0;  // gridDim.x .. threadIdx.x
        for (uint32_t i = 0; i < 12; ++i)
            if (eq(f, names[i])) return i + 1;
        return 0;
    }

    // ---- dead_block_elim (optimize.py:643-675) ---------------------------------
    OCB_HD uint32_t dead_block_elim() {
        if (!k->blocks.n) return 0;
        LabelMap lm;
        lm.build(tmp, m, k->blocks);
        LabelSet reach;
        reach.init(tmp, k->blocks.n * 3 + 4);
        Vec<Str> queue;
        queue.init();
        queue.push(tmp, B(k->blocks[0]).label);
        while (queue.n && !bad()) {
            Str l = queue.back();
            queue.n--;
            if (reach.has(l)) continue;
            reach.add(l);
            int32_t b = lm.get(l);
            if (b >= 0) {
                const Term &t = B((uint32_t)b).term;
                if (t.kind == T_BR) queue.push(tmp, t.t);
                else if (t.kind == T_CBR) {
                    queue.push(tmp, t.t);
                    queue.push(tmp, t.f);
                }
            }
        }
        uint32_t w = 0, removed = 0;
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            if (reach.has(B(k->blocks[i]).label)) k->blocks[w++] = k->blocks[i];
            else removed++;
        }
        k->blocks.n = w;
        return removed;
    }

    // ---- identity_fold (optimize.py:678-776) -----------------------------------
    OCB_HD uint32_t identity_fold() {
        IdArr<uint32_t> dc = def_counts();
        uint32_t n0 = nid();
        IdArr<uint8_t> has;
        has.init(tmp, n0, 0);
        Opnd *src = (Opnd *)tmp.alloc(sizeof(Opnd) * (uint64_t)(n0 ? n0 : 1), 16);
        if (!src || bad()) return 0;
        bool any = false;
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (in.kind != I_BIN || dc.get(did(in)) != 1) continue;
                uint8_t op = in.op;
                bool rz = (op == BO_ADD || op == BO_SUB || op == BO_SHL || op == BO_SHR ||
                           op == BO_XOR || op == BO_OR) && cis(in.b, 0);
                bool lz = (op == BO_ADD || op == BO_XOR || op == BO_OR) && cis(in.a, 0);
                if (rz) {
                    has.set(did(in), 1);
                    src[did(in)] = in.a;
                    any = true;
                } else if (lz) {
                    has.set(did(in), 1);
                    src[did(in)] = in.b;
                    any = true;
                }
            }
        }
        if (!any) return 0;
        IdArr<uint32_t> vis;  // cycle guard of _resolve, stamped per call
        vis.init(tmp, n0, 0);
        uint32_t call_no = 0;
        auto resolve = [&](Opnd o) -> Opnd {
            if (o.k != O_VAL || !has.get(vid(o))) return o;
            ++call_no;
            vis.set(vid(o), call_no);
            Opnd r = src[vid(o)];
            while (r.k == O_VAL && has.get(vid(r))) {
                if (vis.get(vid(r)) == call_no) break;
                vis.set(vid(r), call_no);
                r = src[vid(r)];
            }
            return r;
        };
        uint32_t eliminated = 0;
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            uint32_t w = 0;
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                uint32_t ix = b.insts[ii];
                Inst &in = I(ix);
                if (in.kind == I_BIN && has.get(did(in))) {
                    eliminated++;
                    continue;
                }
                switch (in.kind) {
                case I_BIN:
                case I_CMP:
                case I_STORE:
                    in.a = resolve(in.a);
                    in.b = resolve(in.b);
                    break;
                case I_LOAD:
                case I_CVT: in.a = resolve(in.a); break;
                case I_CALL:
                case I_PRINTF:
                    if (in.args.n) {
                        Vec<Opnd> na = in.args.copy(ar);
                        for (uint32_t q = 0; q < na.n; ++q) na[q] = resolve(na[q]);
                        in.args = na;
                    }
                    break;
                default: break;
                }
                b.insts[w++] = ix;
            }
            b.insts.n = w;
            if (b.term.kind == T_CBR) b.term.v = resolve(b.term.v);
        }
        return eliminated;
    }

    // ---- dead_inst_elim (optimize.py:779-832) ----------------------------------
    // The reference repeats rounds (mark every used id, drop the BinInst /
    // CmpInst / CvtInst whose dest id is unused) until a round drops nothing.
    // Dropping an instruction only ever removes uses, so the instructions that
    // go are exactly those reached by repeatedly dropping one whose dest id has
    // no remaining use: counted uses and a worklist give the same survivors,
    // in the same order, and the same total count, in one pass.
    OCB_HD uint32_t dead_inst_elim() {
        uint32_t n0 = nid();
        IdArr<uint32_t> uses;   // remaining uses per id
        uses.init(tmp, n0, 0);
        IdArr<uint32_t> ndefs;  // removable definitions per id (candidates)
        ndefs.init(tmp, n0, 0);
        if (bad()) return 0;
        auto use = [&](Opnd o) {
            if (o.k == O_VAL) {
                uint32_t id = vid(o);
                uses.set(id, uses.get(id) + 1);
            }
        };
        auto removable = [&](const Inst &in) {
            return in.kind == I_BIN || in.kind == I_CMP || in.kind == I_CVT;
        };
        auto each_operand = [&](const Inst &in, auto f) {
            switch (in.kind) {
            case I_BIN:
            case I_CMP:
            case I_STORE:
                f(in.a);
                f(in.b);
                break;
            case I_CVT:
            case I_LOAD: f(in.a); break;
            default: break;
            }
            if (in.kind == I_ASM) return;  // AsmInst has no attribute the pass reads
            for (uint32_t q = 0; q < in.args.n; ++q) f(in.args[q]);
        };
        uint32_t total = 0;
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            total += b.insts.n;
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                each_operand(in, use);
                if (removable(in)) {
                    uint32_t d = did(in);
                    ndefs.set(d, ndefs.get(d) + 1);
                }
            }
            const Term &t = b.term;
            if (t.kind == T_CBR || t.kind == T_RET) use(t.v);
        }
        // dead[inst index] marks; the worklist holds ids whose uses reached 0
        uint8_t *dead = (uint8_t *)tmp.alloc((uint64_t)m.insts.n + 1, 16);
        uint32_t *work = (uint32_t *)tmp.alloc(4ull * (n0 + 1), 16);
        // removable instructions grouped by dest id (CSR over ids)
        uint32_t *start = (uint32_t *)tmp.alloc(4ull * (n0 + 2), 16);
        uint32_t *list = (uint32_t *)tmp.alloc(4ull * (total + 1), 16);
        if (!dead || !work || !start || !list || bad()) return 0;
        for (uint32_t i = 0; i < m.insts.n; ++i) dead[i] = 0;
        start[0] = 0;
        for (uint32_t id = 0; id < n0; ++id) start[id + 1] = start[id] + ndefs.get(id);
        for (uint32_t id = 0; id < n0; ++id) ndefs.set(id, start[id]);  // fill cursor
        uint32_t nw = 0;
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (!removable(in)) continue;
                uint32_t d = did(in), c = ndefs.get(d);
                list[c] = b.insts[ii];
                ndefs.set(d, c + 1);
            }
        }
        for (uint32_t id = 0; id < n0; ++id)
            if (start[id + 1] > start[id] && uses.get(id) == 0) work[nw++] = id;
        uint32_t eliminated = 0;
        while (nw) {
            uint32_t id = work[--nw];
            for (uint32_t q = start[id]; q < start[id + 1]; ++q) {
                uint32_t ix = list[q];
                if (dead[ix]) continue;
                dead[ix] = 1;
                eliminated++;
                each_operand(I(ix), [&](Opnd o) {
                    if (o.k != O_VAL) return;
                    uint32_t u = vid(o), c = uses.get(u);
                    uses.set(u, c - 1);
                    if (c == 1 && start[u + 1] > start[u]) work[nw++] = u;
                });
            }
        }
        if (eliminated)
            for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
                Block &b = B(k->blocks[bi]);
                uint32_t w = 0;
                for (uint32_t ii = 0; ii < b.insts.n; ++ii)
                    if (!dead[b.insts[ii]]) b.insts[w++] = b.insts[ii];
                b.insts.n = w;
            }
        return eliminated;
    }

    // ---- loops (optimize.py:835-948) -----------------------------------------
    struct Loop {
        Str header, preheader, backedge_src;
        LabelSet body;
    };
    OCB_HD int succs(uint32_t b, Str *out) {
        const Term &t = B(b).term;
        if (t.kind == T_BR) { out[0] = t.t; return 1; }
        if (t.kind == T_CBR) { out[0] = t.t; out[1] = t.f; return 2; }
        return 0;
    }
    // predecessor lists keyed by label (entries in block order, duplicates kept)
    struct Preds {
        uint32_t *start, *cnt, *items;  // by block ordinal of the label's last block
    };
    OCB_HD bool build_preds(LabelMap &lm, IdArr<uint32_t> &ordm, Preds &P) {
        uint32_t nb = k->blocks.n;
        P.start = (uint32_t *)tmp.alloc(4ull * (nb + 1), 16);
        P.cnt = (uint32_t *)tmp.alloc(4ull * (nb + 1), 16);
        P.items = (uint32_t *)tmp.alloc(4ull * (2 * nb + 1), 16);
        if (!P.start || !P.cnt || !P.items) return false;
        for (uint32_t i = 0; i <= nb; ++i) P.cnt[i] = 0;
        Str s[2];
        for (uint32_t i = 0; i < nb; ++i) {
            int ns = succs(k->blocks[i], s);
            for (int q = 0; q < ns; ++q) {
                int32_t b = lm.get(s[q]);
                if (b >= 0) P.cnt[ordm.get((uint32_t)b)]++;
            }
        }
        uint32_t acc = 0;
        for (uint32_t i = 0; i < nb; ++i) {
            P.start[i] = acc;
            acc += P.cnt[i];
            P.cnt[i] = 0;
        }
        for (uint32_t i = 0; i < nb; ++i) {
            int ns = succs(k->blocks[i], s);
            for (int q = 0; q < ns; ++q) {
                int32_t b = lm.get(s[q]);
                if (b >= 0) {
                    uint32_t o = ordm.get((uint32_t)b);
                    P.items[P.start[o] + P.cnt[o]++] = i;  // predecessor's ordinal
                }
            }
        }
        return true;
    }

    OCB_HD bool find_loops(Vec<Loop> &loops) {
        loops.init();
        uint32_t nb = k->blocks.n;
        if (!nb) return true;
        LabelMap lm;
        lm.build(tmp, m, k->blocks);
        IdArr<uint32_t> ordm;
        ordm.init(tmp, m.blocks.n, 0);
        for (uint32_t i = 0; i < nb; ++i) ordm.set(k->blocks[i], i);
        Preds P;
        if (!build_preds(lm, ordm, P)) return false;
        // iterative DFS with the recursion's visiting order
        uint8_t *visited = (uint8_t *)tmp.alloc(nb + 1, 16);
        uint8_t *onst = (uint8_t *)tmp.alloc(nb + 1, 16);
        struct Fr { uint32_t o; uint8_t next; };
        Fr *st = (Fr *)tmp.alloc(sizeof(Fr) * (uint64_t)(nb + 1), 16);
        struct BE { uint32_t src, hdr; };
        Vec<BE> back;
        back.init();
        if (!visited || !onst || !st) return false;
        for (uint32_t i = 0; i < nb; ++i) visited[i] = onst[i] = 0;
        auto ord_of = [&](Str l) -> int32_t {
            int32_t b = lm.get(l);
            return b < 0 ? -1 : (int32_t)ordm.get((uint32_t)b);
        };
        int32_t e = ord_of(B(k->blocks[0]).label);
        uint32_t sp = 0;
        if (e >= 0) {
            visited[e] = 1;
            onst[e] = 1;
            st[sp++] = Fr{(uint32_t)e, 0};
        }
        while (sp) {
            Fr &f = st[sp - 1];
            Str s[2];
            int ns = succs(k->blocks[f.o], s);
            if (f.next >= ns) {
                onst[f.o] = 0;
                sp--;
                continue;
            }
            Str sl = s[f.next++];
            int32_t so = ord_of(sl);
            if (so < 0) continue;
            if (onst[so]) {
                back.push(tmp, BE{f.o, (uint32_t)so});
            } else if (!visited[so]) {
                if (sp >= 990) {  // the reference's recursive DFS hits Python's limit
                    unsup();
                    return false;
                }
                visited[so] = 1;
                onst[so] = 1;
                st[sp++] = Fr{(uint32_t)so, 0};
            }
        }
        // one loop per distinct back edge with a unique preheader
        for (uint32_t bi = 0; bi < back.n; ++bi) {
            bool dup = false;
            for (uint32_t bj = 0; bj < bi && !dup; ++bj)
                dup = back[bj].src == back[bi].src && back[bj].hdr == back[bi].hdr;
            if (dup) continue;
            Loop L;
            L.header = B(k->blocks[back[bi].hdr]).label;
            L.backedge_src = B(k->blocks[back[bi].src]).label;
            L.body.init(tmp, nb + 2);
            L.body.add(L.header);
            Vec<uint32_t> work;
            work.init();
            work.push(tmp, back[bi].src);
            while (work.n) {
                uint32_t c = work.back();
                work.n--;
                Str cl = B(k->blocks[c]).label;
                if (L.body.has(cl)) continue;
                L.body.add(cl);
                int32_t co = ord_of(cl);
                if (co < 0) continue;
                for (uint32_t q = 0; q < P.cnt[co]; ++q) {
                    uint32_t p = P.items[P.start[co] + q];
                    if (!L.body.has(B(k->blocks[p]).label)) work.push(tmp, p);
                }
            }
            int32_t ho = (int32_t)back[bi].hdr;
            uint32_t nnl = 0, pre = 0;
            for (uint32_t q = 0; q < P.cnt[ho]; ++q) {
                uint32_t p = P.items[P.start[ho] + q];
                if (!L.body.has(B(k->blocks[p]).label)) {
                    nnl++;
                    pre = p;
                }
            }
            if (nnl != 1) continue;
            L.preheader = B(k->blocks[pre]).label;
            loops.push(tmp, L);
        }
        return !bad();
    }

    // ---- licm (optimize.py:951-1073) -------------------------------------------
    OCB_HD uint32_t licm() {
        Vec<Loop> loops;
        if (!find_loops(loops) || !loops.n) return 0;
        LabelMap lm;
        lm.build(tmp, m, k->blocks);
        uint32_t nb = k->blocks.n;
        IdArr<uint32_t> idx_of;  // label_to_idx (last wins) by block index
        idx_of.init(tmp, m.blocks.n, 0);
        for (uint32_t i = 0; i < nb; ++i) idx_of.set(k->blocks[i], i);
        IdArr<uint32_t> dc = def_counts();
        IdArr<uint8_t> cond;
        cond.init(tmp, nid(), 0);
        for (uint32_t i = 0; i < nb; ++i) {
            const Term &t = B(k->blocks[i]).term;
            if (t.kind == T_CBR && t.v.k == O_VAL) cond.set(vid(t.v), 1);
        }
        uint32_t total = 0;
        for (uint32_t li = 0; li < loops.n && !bad(); ++li) {
            Loop &L = loops[li];
            int32_t pre = lm.get(L.preheader);
            if (pre < 0) continue;
            size_t mark = tmp.used;
            IdArr<uint8_t> ldef, inv;
            ldef.init(tmp, nid(), 0);
            inv.init(tmp, nid(), 0);
            for (uint32_t i = 0; i < k->blocks.n; ++i) {
                Block &b = B(k->blocks[i]);
                if (!L.body.has(b.label)) continue;
                for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                    const Inst &in = I(b.insts[ii]);
                    if (in.dest >= 0) ldef.set(did(in), 1);
                }
            }
            for (uint32_t i = 0; i < k->blocks.n; ++i) {
                Block &b = B(k->blocks[i]);
                if (L.body.has(b.label)) continue;
                for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                    const Inst &in = I(b.insts[ii]);
                    if (in.dest >= 0 && !ldef.get(did(in))) inv.set(did(in), 1);
                }
            }
            auto is_inv = [&](Opnd o) { return o.k == O_CONST || (o.k == O_VAL && inv.get(vid(o))); };
            // body labels sorted by their block index (label_to_idx; absent -> 0)
            Vec<uint32_t> order;  // block indices of body labels, sorted
            order.init();
            for (uint32_t i = 0; i < nb; ++i) {
                Str l = B(k->blocks[i]).label;
                if (!L.body.has(l)) continue;
                int32_t b = lm.get(l);
                if (b != (int32_t)k->blocks[i]) continue;  // a label counts once
                order.push(tmp, (uint32_t)b);
            }
            // label_to_idx maps a label to its last index; order by that index
            for (uint32_t a = 1; a < order.n; ++a) {
                uint32_t x = order[a];
                int32_t j = (int32_t)a - 1;
                while (j >= 0 && idx_of.get(order[j]) > idx_of.get(x)) {
                    order[j + 1] = order[j];
                    --j;
                }
                order[j + 1] = x;
            }
            bool changed = true;
            while (changed && !bad()) {
                changed = false;
                for (uint32_t oi = 0; oi < order.n; ++oi) {
                    uint32_t bidx = order[oi];
                    Block &b = B(bidx);
                    if (eq(b.label, L.header)) continue;
                    uint32_t w = 0;
                    for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                        uint32_t ix = b.insts[ii];
                        const Inst &in = I(ix);
                        bool hoist = false;
                        if ((in.kind == I_BIN || in.kind == I_CVT) && dc.get(did(in)) == 1 &&
                            !cond.get(did(in))) {
                            hoist = in.kind == I_BIN ? (is_inv(in.a) && is_inv(in.b)) : is_inv(in.a);
                        }
                        if (hoist) {
                            B((uint32_t)pre).insts.push(ar, ix);
                            inv.set(did(in), 1);
                            total++;
                            changed = true;
                            continue;
                        }
                        b.insts[w++] = ix;
                    }
                    b.insts.n = w;
                }
            }
            tmp.used = mark;
        }
        return total;
    }

    // ---- merge_linear_chains (optimize.py:1076-1131) ---------------------------
    // The reference restarts its scan from the first block after every merge.
    // With unique labels a merge leaves every remaining label's predecessor
    // count as it was (A takes over B's terminator, B disappears), so no block
    // before the merge point can start to qualify: one forward scan that
    // re-examines the merging block until it stops qualifying performs the
    // same merges in the same order.  Duplicate labels take the restarting
    // scan.
    OCB_HD bool merge_linear_chains_fast(uint32_t &merged) {
        size_t mark = tmp.used;
        LabelSet seen;
        seen.init(tmp, k->blocks.n + 2);
        for (uint32_t i = 0; i < k->blocks.n; ++i)
            if (!seen.add(B(k->blocks[i]).label)) {
                tmp.used = mark;
                return false;
            }
        LabelMap lm;
        lm.build(tmp, m, k->blocks);
        const uint32_t GONE = 0xffffffffu;
        IdArr<uint32_t> pc;
        pc.init(tmp, m.blocks.n, 0);
        if (!pc.n || !lm.cap) {
            tmp.used = mark;
            return false;
        }
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            Str s[2];
            int ns = succs(k->blocks[i], s);
            for (int q = 0; q < ns; ++q) {
                int32_t b = lm.get(s[q]);
                if (b >= 0) pc.set((uint32_t)b, pc.get((uint32_t)b) + 1);
            }
        }
        uint32_t i = 0, removed = 0;
        while (i < k->blocks.n && !bad()) {
            uint32_t bb = k->blocks[i];
            if (pc.get(bb) != GONE && B(bb).term.kind == T_BR) {
                int32_t tb = lm.get(B(bb).term.t);
                if (tb >= 0 && pc.get((uint32_t)tb) == 1) {
                    uint32_t tn = B((uint32_t)tb).insts.n;
                    for (uint32_t q = 0; q < tn; ++q) B(bb).insts.push(ar, B((uint32_t)tb).insts[q]);
                    B(bb).term = B((uint32_t)tb).term;
                    pc.set((uint32_t)tb, GONE);
                    merged++;
                    removed++;
                    continue;
                }
            }
            ++i;
        }
        if (removed) {
            uint32_t w = 0;
            for (uint32_t j = 0; j < k->blocks.n; ++j)
                if (pc.get(k->blocks[j]) != GONE) k->blocks[w++] = k->blocks[j];
            k->blocks.n = w;
        }
        tmp.used = mark;
        return true;
    }
    OCB_HD uint32_t merge_linear_chains() {
        if (!k->blocks.n) return 0;
        uint32_t merged = 0;
        if (merge_linear_chains_fast(merged)) return merged;
        bool changed = true;
        while (changed && !bad()) {
            changed = false;
            size_t mark = tmp.used;
            LabelMap lm;
            lm.build(tmp, m, k->blocks);
            IdArr<uint32_t> pc;  // pred count by block index of the label's last block
            pc.init(tmp, m.blocks.n, 0);
            for (uint32_t i = 0; i < k->blocks.n; ++i) {
                Str s[2];
                int ns = succs(k->blocks[i], s);
                for (int q = 0; q < ns; ++q) {
                    int32_t b = lm.get(s[q]);
                    if (b >= 0) pc.set((uint32_t)b, pc.get((uint32_t)b) + 1);
                }
            }
            for (uint32_t i = 0; i < k->blocks.n; ++i) {
                uint32_t bb = k->blocks[i];
                const Term &t = B(bb).term;
                if (t.kind != T_BR) continue;
                Str tl = t.t;
                int32_t tb = lm.get(tl);
                if (tb < 0) continue;
                if (pc.get((uint32_t)tb) != 1) continue;
                Block &T = B((uint32_t)tb);
                uint32_t tn = T.insts.n;
                for (uint32_t q = 0; q < tn; ++q) B(bb).insts.push(ar, T.insts[q]);
                B(bb).term = B((uint32_t)tb).term;
                uint32_t w = 0;
                for (uint32_t j = 0; j < k->blocks.n; ++j)
                    if (!eq(B(k->blocks[j]).label, tl)) k->blocks[w++] = k->blocks[j];
                k->blocks.n = w;
                merged++;
                changed = true;
                break;
            }
            tmp.used = mark;
        }
        return merged;
    }

    // ---- thread_empty_blocks (optimize.py:1134-1238) ---------------------------
    OCB_HD uint32_t thread_empty_blocks() {
        if (!k->blocks.n) return 0;
        Str entry = B(k->blocks[0]).label;
        LabelMap lm;
        lm.build(tmp, m, k->blocks);
        LabelSet transparent;
        transparent.init(tmp, k->blocks.n + 2);
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            const Block &b = B(k->blocks[i]);
            if (!eq(b.label, entry) && b.insts.n == 0 && b.term.kind == T_BR) transparent.add(b.label);
        }
        if (!transparent.n) return 0;
        LabelSet visited;
        auto forward = [&](Str l) -> Str {
            visited.init(tmp, k->blocks.n + 2);
            for (;;) {
                if (visited.has(l)) return l;
                int32_t b = lm.get(l);
                if (b < 0) return l;
                if (eq(l, entry)) return l;
                const Block &bb = B((uint32_t)b);
                if (bb.insts.n == 0 && bb.term.kind == T_BR) {
                    visited.add(l);
                    l = bb.term.t;
                } else {
                    return l;
                }
            }
        };
        // fwd map: transparent label -> target (computed before any rewrite)
        struct FE { Str from, to; };
        Vec<FE> fwd;
        fwd.init();
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            const Block &b = B(k->blocks[i]);
            if (!transparent.has(b.label)) continue;
            bool dup = false;
            for (uint32_t q = 0; q < fwd.n && !dup; ++q) dup = eq(fwd[q].from, b.label);
            if (dup) continue;
            size_t mark = tmp.used;
            Str to = forward(b.label);
            tmp.used = mark;
            fwd.push(tmp, FE{b.label, to});
        }
        LabelMap fm;  // from -> index into fwd, via a small open table
        uint32_t fcap = 16;
        while (fcap < 2 * fwd.n + 2) fcap *= 2;
        int32_t *fht = (int32_t *)tmp.alloc(4ull * fcap, 16);
        if (!fht || bad()) return 0;
        for (uint32_t i = 0; i < fcap; ++i) fht[i] = -1;
        for (uint32_t i = 0; i < fwd.n; ++i) {
            uint32_t h = hash(fwd[i].from) & (fcap - 1);
            while (fht[h] >= 0) h = (h + 1) & (fcap - 1);
            fht[h] = (int32_t)i;
        }
        (void)fm;
        auto F = [&](Str l) -> Str {
            uint32_t h = hash(l) & (fcap - 1);
            while (fht[h] >= 0) {
                if (eq(fwd[fht[h]].from, l)) return fwd[fht[h]].to;
                h = (h + 1) & (fcap - 1);
            }
            return l;
        };
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            Term &t = B(k->blocks[i]).term;
            if (t.kind == T_BR) {
                Str nt = F(t.t);
                if (!eq(nt, t.t)) t.t = nt;
            } else if (t.kind == T_CBR) {
                Str ntr = F(t.t), nfa = F(t.f);
                if (!eq(ntr, t.t) || !eq(nfa, t.f)) {
                    if (eq(ntr, nfa)) t = Term{T_BR, onone(), ntr, Str{nullptr, 0}};
                    else {
                        t.t = ntr;
                        t.f = nfa;
                    }
                }
            }
        }
        LabelSet ref;
        ref.init(tmp, 2 * k->blocks.n + 4);
        ref.add(entry);
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            const Term &t = B(k->blocks[i]).term;
            if (t.kind == T_BR) ref.add(t.t);
            else if (t.kind == T_CBR) {
                ref.add(t.t);
                ref.add(t.f);
            }
        }
        uint32_t removed = 0, w = 0;
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            Str l = B(k->blocks[i]).label;
            if (transparent.has(l) && !ref.has(l)) removed++;
            else k->blocks[w++] = k->blocks[i];
        }
        k->blocks.n = w;
        return removed;
    }

    // ---- fold_empty_ret_blocks (optimize.py:1241-1294) -------------------------
    OCB_HD uint32_t fold_empty_ret_blocks() {
        if (!k->blocks.n) return 0;
        Str entry = B(k->blocks[0]).label;
        LabelMap er;  // label -> block with an empty ret (last wins)
        Vec<uint32_t> ers;
        ers.init();
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            const Block &b = B(k->blocks[i]);
            if (eq(b.label, entry)) continue;
            if (b.insts.n == 0 && b.term.kind == T_RET) ers.push(tmp, k->blocks[i]);
        }
        if (!ers.n) return 0;
        er.build(tmp, m, ers);
        uint32_t folded = 0;
        for (uint32_t i = 0; i < k->blocks.n; ++i) {
            Term &t = B(k->blocks[i]).term;
            if (t.kind != T_BR) continue;
            int32_t r = er.get(t.t);
            if (r < 0) continue;
            Opnd rv = B((uint32_t)r).term.v;
            t = Term{T_RET, rv, Str{nullptr, 0}, Str{nullptr, 0}};
            folded++;
        }
        return folded;
    }

    // ---- fma_fuse (optimize.py:1297-1440) ----------------------------------------
    OCB_HD uint32_t fma_fuse() {
        IdArr<uint32_t> dc, uc;
        dc.init(tmp, nid(), 0);
        uc.init(tmp, nid(), 0);
        auto tally = [&](Opnd o) {
            if (o.k == O_VAL) uc.set(vid(o), uc.get(vid(o)) + 1);
        };
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (in.dest >= 0) dc.set(did(in), dc.get(did(in)) + 1);
                switch (in.kind) {
                case I_BIN:
                case I_CMP:
                case I_STORE:
                    tally(in.a);
                    tally(in.b);
                    break;
                case I_CVT:
                case I_LOAD: tally(in.a); break;
                case I_CALL:
                    for (uint32_t q = 0; q < in.args.n; ++q) tally(in.args[q]);
                    break;
                default: break;
                }
            }
            if (b.term.kind == T_CBR) tally(b.term.v);
        }
        IdArr<uint8_t> fus;
        fus.init(tmp, nid(), 0);
        bool any = false;
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (in.kind != I_BIN || in.op != BO_MUL) continue;
                Ty dt = dty(in);
                if (!ty_is_float(dt)) continue;
                if (m.opty(in.a) != dt || m.opty(in.b) != dt) continue;
                if (dc.get(did(in)) != 1 || uc.get(did(in)) != 1) continue;
                fus.set(did(in), 1);
                any = true;
            }
        }
        if (!any) return 0;
        uint32_t fused = 0;
        IdArr<uint32_t> local;  // mul id -> inst index + 1 (last in block wins)
        local.init(tmp, nid(), 0);
        IdArr<uint8_t> fmul;
        fmul.init(tmp, nid(), 0);
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            Vec<uint32_t> lids;
            lids.init();
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (in.kind == I_BIN && in.op == BO_MUL && fus.get(did(in))) {
                    local.set(did(in), b.insts[ii] + 1);
                    lids.push(tmp, did(in));
                }
            }
            if (!lids.n) continue;
            // ADDs consuming a local mul: position -> mul inst (0 = none)
            uint32_t *fz = (uint32_t *)tmp.alloc(4ull * (b.insts.n + 1), 16);
            if (!fz) return fused;
            bool anyf = false;
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                fz[ii] = 0;
                const Inst &in = I(b.insts[ii]);
                if (in.kind != I_BIN || in.op != BO_ADD || !ty_is_float(dty(in))) continue;
                if (in.a.k == O_VAL && local.get(vid(in.a))) fz[ii] = local.get(vid(in.a)) * 2;
                else if (in.b.k == O_VAL && local.get(vid(in.b))) fz[ii] = local.get(vid(in.b)) * 2 + 1;
                if (fz[ii]) anyf = true;
            }
            if (anyf) {
                for (uint32_t ii = 0; ii < b.insts.n; ++ii)
                    if (fz[ii]) fmul.set(did(I(fz[ii] / 2 - 1)), 1);
                uint32_t w = 0;
                for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                    uint32_t ix = b.insts[ii];
                    const Inst &in = I(ix);
                    if (in.kind == I_BIN && in.op == BO_MUL && fmul.get(did(in))) continue;
                    if (fz[ii]) {
                        const Inst &mul = I(fz[ii] / 2 - 1);
                        Opnd addend = (fz[ii] & 1) ? in.a : in.b;
                        bool dbl = ty_scalar(dty(in)) == S_DOUBLE;
                        Inst c = mk_inst(I_CALL, 0, in.dest, onone(), onone());
                        c.func = S(dbl ? "fma" : "fmaf");
                        c.args.push(ar, mul.a);
                        c.args.push(ar, mul.b);
                        c.args.push(ar, addend);
                        b.insts[w++] = add_inst(c);
                        fused++;
                        continue;
                    }
                    b.insts[w++] = ix;
                }
                b.insts.n = w;
            }
            // local_muls is per block
            for (uint32_t q = 0; q < lids.n; ++q) local.set(lids[q], 0);
        }
        return fused;
    }

    // ---- unroll (unroll.py) --------------------------------------------------------
    struct Carried { uint32_t cid; uint32_t cval; Opnd nval; };
    struct Sec { uint32_t cid; uint32_t cval; pyint init, step; };
    struct ULoop {
        uint32_t cond_b, body_b, inc_b, exit_b;
        uint32_t ind;  // induction value index
        pyint init, step, trip;
        Vec<Carried> carried;
        Vec<Sec> sec;
    };
    // int(const.value) for the unroller's bound/init/step reads.  Floats
    // beyond the kept range saturate (they only ever fail the trip-count
    // checks); `sat_seen` records it so a loop that would still be unrolled
    // with such a value is declined.  int() of NaN raises ValueError and of
    // an infinity OverflowError (unroll.py:84-109), ending the compile.
    bool sat_seen = false;
    OCB_HD bool opnd_int(Opnd o, pyint &out) {
        PyVal v = cv(o);
        if (pv_to_int(v, out)) return true;
        if (!is_finite(v.f)) {
            m.raises = v.f != v.f ? 1 : 2;  // OCB_TU_RAISES_VALUEERROR / _OVERFLOW
            return false;
        }
        out = v.f > 0 ? PYINT_LIM : -PYINT_LIM;
        sat_seen = true;
        return true;
    }
    // The constant operand a definition of _resolve_const_value's patterns
    // reads (unroll.py:30-45), or onone(): CvtInst of a Const, or
    // BinInst ADD of a Const and a zero Const (in that order of checks).
    OCB_HD Opnd const_def_operand(const Inst &in) const {
        if (in.kind == I_CVT && in.a.k == O_CONST) return in.a;
        if (in.kind == I_BIN && in.op == BO_ADD) {
            if (in.b.k == O_CONST && cis(in.b, 0)) {
                if (in.a.k == O_CONST) return in.a;
            } else if (in.a.k == O_CONST && cis(in.a, 0)) {
                if (in.b.k == O_CONST) return in.b;
            }
        }
        return onone();
    }
    // id -> index + 1 of the first instruction (block order) that defines the
    // id with one of those patterns; built once per find_unrollable call, so
    // each lookup is O(1) instead of a scan of the kernel
    IdArr<uint32_t> const_def;
    OCB_HD void build_const_defs() {
        const_def.init(tmp, nid(), 0);
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (in.dest < 0) continue;
                uint32_t d = did(in);
                if (const_def.get(d) == 0 && const_def_operand(in).k == O_CONST)
                    const_def.set(d, b.insts[ii] + 1);
            }
        }
    }
    // _resolve_const_value (unroll.py:21-45): the first definition of `id`
    // that matches a pattern decides
    OCB_HD bool resolve_const_value(uint32_t id, pyint &out) {
        uint32_t ix = const_def.get(id);
        if (!ix) return false;
        return opnd_int(const_def_operand(I(ix - 1)), out);
    }
    OCB_HD void carried_put(Vec<Carried> &c, uint32_t cid, uint32_t cval, Opnd nval) {
        for (uint32_t i = 0; i < c.n; ++i)
            if (c[i].cid == cid) {
                c[i].cval = cval;
                c[i].nval = nval;
                return;
            }
        c.push(tmp, Carried{cid, cval, nval});
    }
    OCB_HD bool find_unrollable(Vec<ULoop> &out) {
        out.init();
        LabelMap lm;
        lm.build(tmp, m, k->blocks);
        build_const_defs();
        // `add` definitions per value id in block-then-instruction order: the
        // init scans below visit a value's definitions only, in the order
        // the reference's scans over every block reach them.
        uint32_t nv = nid();
        uint32_t *astart = (uint32_t *)tmp.alloc(4ull * (nv + 2), 16);
        if (!astart) return false;
        for (uint32_t q = 0; q <= nv + 1; ++q) astart[q] = 0;
        uint32_t nadd = 0;
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (in.kind != I_BIN || in.op != BO_ADD || in.dest < 0) continue;
                uint32_t d = did(in);
                if (d < nv) {
                    astart[d + 1]++;
                    nadd++;
                }
            }
        }
        for (uint32_t q = 0; q < nv; ++q) astart[q + 1] += astart[q];
        uint32_t *aref_b = (uint32_t *)tmp.alloc(4ull * (nadd + 1), 16);
        uint32_t *aref_i = (uint32_t *)tmp.alloc(4ull * (nadd + 1), 16);
        uint32_t *afill = (uint32_t *)tmp.alloc(4ull * (nv + 1), 16);
        if (!aref_b || !aref_i || !afill) return false;
        for (uint32_t q = 0; q < nv; ++q) afill[q] = astart[q];
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                if (in.kind != I_BIN || in.op != BO_ADD || in.dest < 0) continue;
                uint32_t d = did(in);
                if (d >= nv) continue;
                aref_b[afill[d]] = bi;
                aref_i[afill[d]] = b.insts[ii];
                afill[d]++;
            }
        }
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            uint32_t cb = k->blocks[bi];
            sat_seen = false;
            if (B(cb).term.kind != T_CBR) continue;
            int32_t cmpi = -1;
            for (uint32_t ii = 0; ii < B(cb).insts.n; ++ii)
                if (I(B(cb).insts[ii]).kind == I_CMP) cmpi = (int32_t)B(cb).insts[ii];
            if (cmpi < 0) continue;
            const Inst cmp = I((uint32_t)cmpi);
            bool have = false;
            pyint bound = 0;
            Opnd ind = onone();
            if (cmp.op == CO_LT && cmp.b.k == O_CONST && cmp.a.k == O_VAL) {
                if (!opnd_int(cmp.b, bound)) return false;
                ind = cmp.a;
                have = true;
            } else if (cmp.op == CO_LT && cmp.b.k == O_VAL && cmp.a.k == O_VAL) {
                pyint r;
                if (resolve_const_value(vid(cmp.b), r)) {
                    bound = r;
                    ind = cmp.a;
                    have = true;
                }
                if (bad()) return false;
            } else if (cmp.op == CO_GT && cmp.a.k == O_CONST && cmp.b.k == O_VAL) {
                if (!opnd_int(cmp.a, bound)) return false;
                ind = cmp.b;
                have = true;
            } else if (cmp.op == CO_LE && cmp.b.k == O_CONST && cmp.a.k == O_VAL) {
                if (!opnd_int(cmp.b, bound)) return false;
                bound += 1;
                ind = cmp.a;
                have = true;
            } else if (cmp.op == CO_LE && cmp.b.k == O_VAL && cmp.a.k == O_VAL) {
                pyint r;
                if (resolve_const_value(vid(cmp.b), r)) {
                    bound = r + 1;
                    ind = cmp.a;
                    have = true;
                }
                if (bad()) return false;
            } else if (cmp.op == CO_GE && cmp.a.k == O_CONST && cmp.b.k == O_VAL) {
                if (!opnd_int(cmp.a, bound)) return false;
                bound += 1;
                ind = cmp.b;
                have = true;
            }
            if (!have || ind.k != O_VAL) continue;
            const Term &ct = B(cb).term;
            if (!(ct.v.k == O_VAL && vid(ct.v) == did(cmp))) continue;
            if (bound <= 0 || bound > 64) continue;
            int32_t body = lm.get(ct.t), ex = lm.get(ct.f);
            if (body < 0 || ex < 0) continue;
            if (B((uint32_t)body).term.kind != T_BR) continue;
            int32_t inc = lm.get(B((uint32_t)body).term.t);
            if (inc < 0) continue;
            if (B((uint32_t)inc).term.kind != T_BR) continue;
            if (!eq(B((uint32_t)inc).term.t, B(cb).label)) continue;
            ULoop L;
            L.cond_b = cb;
            L.body_b = (uint32_t)body;
            L.inc_b = (uint32_t)inc;
            L.exit_b = (uint32_t)ex;
            L.ind = ind.x;
            L.carried.init();
            L.sec.init();
            uint32_t chk[2] = {(uint32_t)body, (uint32_t)inc};
            for (int q = 0; q < 2; ++q) {
                Block &b = B(chk[q]);
                for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                    const Inst &in = I(b.insts[ii]);
                    if (in.kind != I_BIN || in.op != BO_ADD) continue;
                    if (in.b.k == O_CONST && cis(in.b, 0)) {
                        if (in.a.k == O_VAL) carried_put(L.carried, did(in), (uint32_t)in.dest, in.a);
                    } else if (in.a.k == O_CONST && cis(in.a, 0)) {
                        if (in.b.k == O_VAL) carried_put(L.carried, did(in), (uint32_t)in.dest, in.b);
                    }
                }
            }
            Str ll[3] = {B(cb).label, B((uint32_t)body).label, B((uint32_t)inc).label};
            auto in_loop = [&](Str l) { return eq(l, ll[0]) || eq(l, ll[1]) || eq(l, ll[2]); };
            uint32_t ind_id = vid(ind);
            pyint init = 0;
            for (uint32_t ap = ind_id < nv ? astart[ind_id] : 0;
                 ind_id < nv && ap < astart[ind_id + 1]; ++ap) {
                Block &b = B(k->blocks[aref_b[ap]]);
                if (in_loop(b.label)) continue;
                {
                    const Inst &in = I(aref_i[ap]);
                    pyint z;
                    if (in.b.k == O_CONST) {
                        if (!opnd_int(in.b, z)) return false;
                        if (z == 0) {
                            if (in.a.k == O_CONST && !opnd_int(in.a, init)) return false;
                            continue;
                        }
                    }
                    if (in.b.k != O_CONST || z != 0) {
                        if (in.a.k == O_CONST) {
                            if (!opnd_int(in.a, z)) return false;
                            if (z == 0 && in.b.k == O_CONST && !opnd_int(in.b, init)) return false;
                        }
                    }
                }
            }
            pyint step = 1;
            Block &ib = B((uint32_t)inc);
            for (uint32_t ii = 0; ii < ib.insts.n; ++ii) {
                const Inst &in = I(ib.insts[ii]);
                if (in.kind != I_BIN || in.op != BO_ADD) continue;
                pyint s;
                if (in.a.k == O_VAL && vid(in.a) == ind_id && in.b.k == O_CONST) {
                    if (!opnd_int(in.b, s)) return false;
                    if (s > 0) step = s;
                } else if (in.b.k == O_VAL && vid(in.b) == ind_id && in.a.k == O_CONST) {
                    if (!opnd_int(in.a, s)) return false;
                    if (s > 0) step = s;
                }
            }
            pyint span = bound - init;
            if (span <= 0) continue;
            if (span % step != 0) continue;
            pyint trip = span / step;
            if (trip > 64) continue;
            // secondary induction variables
            for (uint32_t ci = 0; ci < L.carried.n; ++ci) {
                const Carried &c = L.carried[ci];
                if (c.cid == ind_id) continue;
                if (c.nval.k != O_VAL) continue;
                int32_t di = -1;
                for (uint32_t ii = 0; ii < ib.insts.n; ++ii) {
                    const Inst &in = I(ib.insts[ii]);
                    if (in.dest >= 0 && did(in) == vid(c.nval)) di = (int32_t)ib.insts[ii];
                }
                if (di < 0 || I((uint32_t)di).kind != I_BIN) continue;
                const Inst &dfi = I((uint32_t)di);
                if (dfi.op != BO_ADD && dfi.op != BO_SUB) continue;
                pyint sstep;
                if (dfi.a.k == O_VAL && vid(dfi.a) == c.cid && dfi.b.k == O_CONST) {
                    pyint raw;
                    if (!opnd_int(dfi.b, raw)) return false;
                    sstep = dfi.op == BO_SUB ? -raw : raw;
                } else if (dfi.op == BO_ADD && dfi.b.k == O_VAL && vid(dfi.b) == c.cid &&
                           dfi.a.k == O_CONST) {
                    if (!opnd_int(dfi.a, sstep)) return false;
                } else {
                    continue;
                }
                bool have_init = false;
                pyint sinit = 0;
                for (uint32_t ap = c.cid < nv ? astart[c.cid] : 0;
                     c.cid < nv && ap < astart[c.cid + 1]; ++ap) {
                    Block &b = B(k->blocks[aref_b[ap]]);
                    if (in_loop(b.label)) continue;
                    {
                        const Inst &in = I(aref_i[ap]);
                        pyint z;
                        if (in.b.k == O_CONST) {
                            if (!opnd_int(in.b, z)) return false;
                            if (z == 0) {
                                if (in.a.k == O_CONST) {
                                    if (!opnd_int(in.a, sinit)) return false;
                                    have_init = true;
                                }
                                continue;
                            }
                        }
                        if (in.a.k == O_CONST) {
                            if (!opnd_int(in.a, z)) return false;
                            if (z == 0 && in.b.k == O_CONST) {
                                if (!opnd_int(in.b, sinit)) return false;
                                have_init = true;
                            }
                        }
                    }
                }
                if (have_init) {
                    bool found = false;
                    for (uint32_t q = 0; q < L.sec.n; ++q)
                        if (L.sec[q].cid == c.cid) {
                            L.sec[q] = Sec{c.cid, c.cval, sinit, sstep};
                            found = true;
                        }
                    if (!found) L.sec.push(tmp, Sec{c.cid, c.cval, sinit, sstep});
                }
            }
            L.init = init;
            L.step = step;
            L.trip = trip;
            if (sat_seen) {  // a saturated value reached an unrolled loop
                unsup();
                return false;
            }
            out.push(tmp, L);
        }
        return !bad();
    }

    OCB_HD uint32_t unroll_loops(uint32_t max_unroll) {
        Vec<ULoop> loops;
        if (!find_unrollable(loops)) return 0;
        uint32_t count = 0;
        Vec<Str> gone;  // labels of the unrolled loops' body and increment blocks
        gone.init();
        // Id-indexed tables shared by every loop of this call, sized for the
        // values all of them can add, filled once and told apart by stamps:
        // remap entries by iteration (gen), carried remaps by loop, the
        // iteration's new dests by iteration.
        uint64_t cap64 = (uint64_t)nid() + 1024;
        for (uint32_t li = 0; li < loops.n; ++li)
            if (loops[li].trip <= (pyint)max_unroll)
                cap64 += (uint64_t)loops[li].trip * (B(loops[li].body_b).insts.n + 2) + 8;
        if (cap64 > 0x7FFFFFFFull) { unsup(); return 0; }
        uint32_t cap = (uint32_t)cap64;
        IdArr<uint32_t> st;     // iteration stamp of rm[id]
        st.init(tmp, cap, 0xFFFFFFFFu);
        Opnd *rm = (Opnd *)tmp.alloc(sizeof(Opnd) * (uint64_t)cap, 16);
        IdArr<uint32_t> cstamp;  // loop stamp of cval[id]
        cstamp.init(tmp, cap, 0xFFFFFFFFu);
        uint32_t *cval = (uint32_t *)tmp.alloc(4ull * cap, 16);
        IdArr<uint32_t> nstamp;  // iteration stamp of nval[id]
        nstamp.init(tmp, cap, 0xFFFFFFFFu);
        uint32_t *nval = (uint32_t *)tmp.alloc(4ull * cap, 16);
        if (!rm || !cval || !nval || bad()) return 0;
        uint32_t gen = 0;
        for (uint32_t li = 0; li < loops.n && !bad(); ++li) {
            ULoop &L = loops[li];
            if (L.trip > (pyint)max_unroll) continue;
            // carried_remap: id -> value index + 1 (0: none)
            auto cst_get = [&](uint32_t id) -> uint32_t { return cstamp.get(id) == li ? cval[id] : 0u; };
            auto cst_set = [&](uint32_t id, uint32_t v) {
                if (!cstamp.set(id, li)) { unsup(); return; }
                cval[id] = v;
            };
            Vec<uint32_t> all;
            all.init();
            Ty ind_ty = m.vals[L.ind].ty;
            uint32_t ind_id = m.vals[L.ind].id;
            for (pyint it = 0; it < L.trip; ++it) {
                uint32_t itn = (uint32_t)it;
                const uint32_t g = gen++;
                auto rset = [&](uint32_t id, Opnd o) {
                    if (!st.set(id, g)) { unsup(); return; }
                    rm[id] = o;
                };
                // remap = dict(carried_remap)
                for (uint32_t ci = 0; ci < L.carried.n; ++ci) {
                    uint32_t v = cst_get(L.carried[ci].cid);
                    if (v) rset(L.carried[ci].cid, ov(v - 1));
                }
                rset(ind_id, cint(ind_ty, L.init + L.step * it));
                for (uint32_t q = 0; q < L.sec.n; ++q)
                    rset(L.sec[q].cid, cint(m.vals[L.sec[q].cval].ty, L.sec[q].init + L.sec[q].step * it));
                auto R = [&](Opnd o) -> Opnd {
                    if (o.k == O_VAL && st.get(vid(o)) == g) return rm[vid(o)];
                    return o;
                };
                // iter_new_vals: body dest id -> new dest (value index + 1)
                auto inv_get = [&](uint32_t id) -> uint32_t { return nstamp.get(id) == g ? nval[id] : 0u; };
                Block &bb = B(L.body_b);
                for (uint32_t ii = 0; ii < bb.insts.n; ++ii) {
                    const Inst in = I(bb.insts[ii]);
                    Inst ni = in;
                    bool has_new_dest = false;
                    switch (in.kind) {
                    case I_BIN:
                    case I_CMP:
                        ni.a = R(in.a);
                        ni.b = R(in.b);
                        has_new_dest = true;
                        break;
                    case I_LOAD:
                    case I_CVT:
                        ni.a = R(in.a);
                        has_new_dest = true;
                        break;
                    case I_STORE:
                        ni.a = R(in.a);
                        ni.b = R(in.b);
                        break;
                    case I_CALL:
                        if (eq(in.func, "__syncthreads")) break;
                        ni.args = in.args.copy(ar);
                        for (uint32_t q = 0; q < ni.args.n; ++q) ni.args[q] = R(ni.args[q]);
                        has_new_dest = in.dest >= 0;
                        break;
                    case I_PRINTF:
                        ni.args = in.args.copy(ar);
                        for (uint32_t q = 0; q < ni.args.n; ++q) ni.args[q] = R(ni.args[q]);
                        break;
                    default: break;
                    }
                    if (has_new_dest) {
                        const Value &ov_ = m.vals[(uint32_t)in.dest];
                        Str nm = cat(ar, ov_.name, S("_u"), utoa(ar, itn));
                        uint32_t nd = new_value(nm, ov_.ty);
                        ni.dest = (int32_t)nd;
                        rset(ov_.id, ov(nd));
                        if (!nstamp.set(ov_.id, g)) { unsup(); return count; }
                        nval[ov_.id] = nd + 1;
                    }
                    all.push(ar, add_inst(ni));
                }
                for (uint32_t ci = 0; ci < L.carried.n; ++ci) {
                    uint32_t v = inv_get(L.carried[ci].cid);
                    if (v) cst_set(L.carried[ci].cid, v);
                }
                if (bad()) return count;
            }
            for (uint32_t ci = 0; ci < L.carried.n; ++ci) {
                uint32_t v = cst_get(L.carried[ci].cid);
                if (!v) continue;
                Ty cty = m.vals[L.carried[ci].cval].ty;
                Opnd z = ty_is_float(cty) ? cflt(cty, 0.0) : cint(cty, 0);
                all.push(ar, add_inst(mk_inst(I_BIN, BO_ADD, (int32_t)L.carried[ci].cval, ov(v - 1), z)));
            }
            B(L.cond_b).insts = all;
            set_br(L.cond_b, B(L.exit_b).label);
            // the loop's body and increment blocks leave the kernel (by label);
            // the filter runs once for every unrolled loop of this call, which
            // removes the same blocks as a filter per loop
            gone.push(tmp, B(L.body_b).label);
            gone.push(tmp, B(L.inc_b).label);
            count++;
        }
        if (count) {
            LabelSet gs;
            gs.init(tmp, gone.n + 8);
            for (uint32_t q = 0; q < gone.n; ++q) gs.add(gone[q]);
            uint32_t w = 0;
            for (uint32_t j = 0; j < k->blocks.n; ++j)
                if (!gs.has(B(k->blocks[j]).label)) k->blocks[w++] = k->blocks[j];
            k->blocks.n = w;
        }
        return count;
    }

    // ---- optimize() schedule (optimize.py:1493-1582) ------------------------------
#define OCB_PASS(call) (reset_tmp(), (call))
    OCB_HD void run() {
        for (int r = 0; r < 8 && !bad(); ++r) {
            uint32_t n = OCB_PASS(unroll_loops(16));
            if (n == 0) break;
            OCB_PASS(constant_fold());
            OCB_PASS(dead_block_elim());
            OCB_PASS(dead_inst_elim());
            OCB_PASS(merge_linear_chains());
        }
        OCB_PASS(constant_fold());
        OCB_PASS(cse());
        OCB_PASS(dead_block_elim());
        OCB_PASS(identity_fold());
        OCB_PASS(constant_fold());
        OCB_PASS(dead_inst_elim());
        OCB_PASS(licm());
        OCB_PASS(fma_fuse());
        OCB_PASS(cse());
        OCB_PASS(identity_fold());
        OCB_PASS(constant_fold());
        OCB_PASS(dead_inst_elim());
        OCB_PASS(thread_empty_blocks());
        OCB_PASS(fold_empty_ret_blocks());
        for (int r = 0; r < 8 && !bad(); ++r) {
            uint32_t a = OCB_PASS(dead_block_elim());
            uint32_t b = OCB_PASS(dead_inst_elim());
            uint32_t c = OCB_PASS(thread_empty_blocks());
            if (a == 0 && b == 0 && c == 0) break;
        }
        // The reference runs this loop until a round reports no change; the
        // counts include no-op refolds of `add c, 0`, so it usually runs all 8
        // rounds.  Every pass is a function of the IR's content (and the next
        // value id), so a round that leaves the content unchanged is a fixed
        // point: the remaining rounds cannot change anything and are skipped.
        // The content before the first round counts too: when the first round
        // leaves it unchanged, every later round repeats it.
        uint64_t fp_prev[2] = {0, 0};
        fingerprint(fp_prev);
        bool have_fp = true;
        for (int r = 0; r < 8 && !bad(); ++r) {
            uint32_t n = 0;
            n += OCB_PASS(unroll_loops(16));
            n += OCB_PASS(constant_fold());
            n += OCB_PASS(cse());
            n += OCB_PASS(identity_fold());
            n += OCB_PASS(fma_fuse());
            n += OCB_PASS(dead_inst_elim());
            n += OCB_PASS(dead_block_elim());
            n += OCB_PASS(thread_empty_blocks());
            n += OCB_PASS(fold_empty_ret_blocks());
            if (n == 0) break;
            OCB_PASS(merge_linear_chains());
            uint64_t fp[2];
            fingerprint(fp);
            if (have_fp && fp[0] == fp_prev[0] && fp[1] == fp_prev[1]) break;
            fp_prev[0] = fp[0];
            fp_prev[1] = fp[1];
            have_fp = true;
        }
        reset_tmp();
    }

    // The pass schedule of a recursive device function's body
    // (optimize.py:1606-1627); the final loop stops at the first pass of a
    // round that changed something, as `and` does there.
    OCB_HD void run_devfn() {
        OCB_PASS(unroll_loops(16));
        OCB_PASS(constant_fold());
        OCB_PASS(cse());
        OCB_PASS(dead_block_elim());
        OCB_PASS(identity_fold());
        OCB_PASS(constant_fold());
        OCB_PASS(dead_inst_elim());
        OCB_PASS(licm());
        OCB_PASS(fma_fuse());
        OCB_PASS(cse());
        OCB_PASS(identity_fold());
        OCB_PASS(constant_fold());
        OCB_PASS(dead_inst_elim());
        OCB_PASS(thread_empty_blocks());
        OCB_PASS(fold_empty_ret_blocks());
        for (int r = 0; r < 8 && !bad(); ++r) {
            if (OCB_PASS(dead_block_elim()) != 0) continue;
            if (OCB_PASS(dead_inst_elim()) != 0) continue;
            if (OCB_PASS(thread_empty_blocks()) != 0) continue;
            if (OCB_PASS(fold_empty_ret_blocks()) != 0) continue;
            break;
        }
        reset_tmp();
    }

    // Content hash of the kernel's IR: blocks (labels, order, terminators),
    // instructions with their operands (values by record, constants by type
    // and Python value) and the next value id.  A value record (id, type,
    // name) is immutable and new ones advance the next value id, so equal
    // hashes across a round still mean equal content.
    OCB_HD void fingerprint(uint64_t out[2]) {
        uint64_t h1 = 1469598103934665603ull, h2 = 0x9E3779B97F4A7C15ull;
        auto mix = [&](uint64_t v) {
            h1 = (h1 ^ v) * 1099511628211ull;
            h2 = (h2 + v + (h2 << 6) + (h2 >> 2)) * 0xff51afd7ed558ccdull;
        };
        auto mix_str = [&](Str s_) {
            mix(s_.n);
            for (uint32_t i = 0; i < s_.n; ++i) mix((uint8_t)s_.p[i]);
        };
        auto mix_op = [&](Opnd o) {
            mix(o.k);
            if (o.k == O_VAL) {
                mix(o.x);  // value records are never changed once made
            } else if (o.k == O_CONST) {
                const Const &c = m.consts[o.x];
                mix(c.ty);
                mix(c.pyfloat);
                if (c.pyfloat) {
                    uint64_t b;
                    memcpy(&b, &c.f, 8);
                    mix(b);
                } else {
                    mix((uint64_t)c.i);
                    mix((uint64_t)((unsigned __int128)c.i >> 64));
                }
            }
        };
        mix(k->next_id);
        mix(k->blocks.n);
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            const Block &b = B(k->blocks[bi]);
            mix_str(b.label);
            mix(b.insts.n);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                mix(in.kind);
                mix(in.op);
                if (in.dest >= 0) mix_op(ov((uint32_t)in.dest));
                else mix(0xFFFF);
                mix_op(in.a);
                mix_op(in.b);
                mix_op(in.c);
                mix_str(in.func);
                mix(in.pidx);
                mix(in.args.n);
                for (uint32_t q = 0; q < in.args.n; ++q) mix_op(in.args[q]);
            }
            mix(b.term.kind);
            mix_op(b.term.v);
            mix_str(b.term.t);
            mix_str(b.term.f);
        }
        out[0] = h1;
        out[1] = h2;
    }
#undef OCB_PASS
};

// optimize(module) for the kernels of a TU
OCB_HD inline void optimize_module(Module &m, Arena &tmp) {
    Opt o(m, tmp);
    for (uint32_t ki = 0; ki < m.kernels.n && !o.bad(); ++ki) {
        o.k = &m.kernels[ki];
        o.run();
    }
    for (uint32_t fi = 0; fi < m.funcs.n && !o.bad(); ++fi) {
        o.k = &m.funcs[fi];
        o.run_devfn();
    }
}

}  // namespace cc
}  // namespace ocb
