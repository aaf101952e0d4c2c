// PTX emitter, kernel level: emit.py:648-1126 (emit_kernel: allocation, the
// body, the five text peepholes, declarations, initialisers), the if-convert
// gate of optimizer/if_convert.py, ir_to_ptx (:3126-3196) and the --emit-ptx
// module text of __main__.py:60-85.
#pragma once
#include "cc_emit_inst.cuh"
#include "cc_dump.cuh"

namespace ocb {
namespace cc {

// ---- line patterns of the peepholes ----------------------------------------------
// `\s+shl\.b32\s+(%\w+),\s*(%\w+),\s*(\d+);` (re.match: anchored at the start only)
OCB_HD inline bool pat_shl(Str l, Str &d, Str &s, Str &n) {
    Cur c{l, 0};
    return c.ws1() && c.lit("shl.b32") && c.ws1() && c.reg(d) && c.lit(",") && (c.ws0(), true) &&
           c.reg(s) && c.lit(",") && (c.ws0(), true) && c.digits(n) && c.lit(";");
}
// `\s+cvt\.s64\.s32\s+(%\w+),\s*(%\w+);`
OCB_HD inline bool pat_cvt64(Str l, Str &d, Str &s) {
    Cur c{l, 0};
    return c.ws1() && c.lit("cvt.s64.s32") && c.ws1() && c.reg(d) && c.lit(",") && (c.ws0(), true) &&
           c.reg(s) && c.lit(";");
}
// `^(\s+)(ld\.\S+)\s+(%\w+),\s*(\[.+\]);$`
OCB_HD inline bool pat_ld(Str l, Str &indent, Str &dst) {
    Cur c{l, 0};
    uint32_t i0 = c.i;
    if (!c.ws1()) return false;
    indent = Str{l.p, c.i - i0};
    if (!c.lit("ld.")) return false;
    // \S+ then \s+ : the maximal non-space run (backtracking cannot help)
    Str tail;
    if (!c.nonws(tail)) return false;
    if (!c.ws1()) return false;
    if (!c.reg(dst) || !c.lit(",")) return false;
    c.ws0();
    if (c.ch() != '[') return false;
    // `\[.+\];$`: ends with "];" and something between
    if (l.n < c.i + 4) return false;
    if (l.p[l.n - 1] != ';' || l.p[l.n - 2] != ']') return false;
    return l.n - 2 > c.i + 1;
}
// `^\s+@(%\w+)\s+mov\.\w+\s+%\w+,\s*(%\w+);$`
OCB_HD inline bool pat_pmov_reg(Str l, Str &pred, Str &src) {
    Cur c{l, 0};
    Str t, d;
    if (!(c.ws1() && c.lit("@") && c.reg(pred) && c.ws1() && c.lit("mov.") && c.word(t) && c.ws1() &&
          c.reg(d) && c.lit(",")))
        return false;
    c.ws0();
    return c.reg(src) && c.lit(";") && c.end();
}
// `^\s+@!(%\w+)\s+mov\.\w+\s+(%\w+),\s*\S+;$`  (dest captured)
OCB_HD inline bool pat_nmov_any(Str l, Str &pred, Str &dst, Str &val) {
    Cur c{l, 0};
    Str t;
    if (!(c.ws1() && c.lit("@!") && c.reg(pred) && c.ws1() && c.lit("mov.") && c.word(t) && c.ws1() &&
          c.reg(dst) && c.lit(",")))
        return false;
    c.ws0();
    // \S+;$ : the rest is non-space and ends with ';' (at least one char before)
    uint32_t st = c.i;
    if (l.n < st + 2 || l.p[l.n - 1] != ';') return false;
    for (uint32_t q = st; q < l.n; ++q)
        if (is_wsc(l.p[q])) return false;
    val = Str{l.p + st, l.n - 1 - st};
    return true;
}
// `^(\s+)@(%\w+)\s+mov\.(\w+)\s+(%\w+),\s*(%\w+);$`
OCB_HD inline bool pat_pmov(Str l, Str &indent, Str &pred, Str &ty, Str &dst, Str &src) {
    Cur c{l, 0};
    if (!c.ws1()) return false;
    indent = Str{l.p, c.i};
    if (!(c.lit("@") && c.reg(pred) && c.ws1() && c.lit("mov.") && c.word(ty) && c.ws1() && c.reg(dst) &&
          c.lit(",")))
        return false;
    c.ws0();
    return c.reg(src) && c.lit(";") && c.end();
}
// `^\s+mov\.\w+\s+(%\w+),\s*(%\w+);$`
OCB_HD inline bool pat_mov_full(Str l, Str &dst, Str &src) {
    Cur c{l, 0};
    Str t;
    if (!(c.ws1() && c.lit("mov.") && c.word(t) && c.ws1() && c.reg(dst) && c.lit(","))) return false;
    c.ws0();
    return c.reg(src) && c.lit(";") && c.end();
}
// `\s+mov\.b\d+\s+(%\w+),\s*(%\w+);` (re.match; trailing text allowed)
OCB_HD inline bool pat_movb(Str l, Str &dst, Str &src) {
    Cur c{l, 0};
    Str n;
    if (!(c.ws1() && c.lit("mov.b") && c.digits(n) && c.ws1() && c.reg(dst) && c.lit(","))) return false;
    c.ws0();
    return c.reg(src) && c.lit(";");
}
// `\s+\S+\s+(%\w+),` -> the destination register of an instruction line
OCB_HD inline bool pat_dest(Str l, Str &dst) {
    Cur c{l, 0};
    Str op;
    if (!c.ws1() || !c.nonws(op) || !c.ws1()) return false;
    return c.reg(dst) && c.lit(",");
}
// `%([a-zA-Z]+)\d` -> register class
OCB_HD inline Str reg_class(Str r) {
    if (r.n < 2 || r.p[0] != '%') return Str{"", 0};
    uint32_t j = 1;
    while (j < r.n && ((r.p[j] >= 'a' && r.p[j] <= 'z') || (r.p[j] >= 'A' && r.p[j] <= 'Z'))) ++j;
    if (j == 1 || j >= r.n || !is_dg(r.p[j])) return Str{"", 0};
    return Str{r.p + 1, j - 1};
}
// `\s+(?:@!?\S+\s+)?bra(?:\.U)?\s+(\w+);`
OCB_HD inline bool pat_bra(Str l, Str &tgt) {
    Cur c{l, 0};
    if (!c.ws1()) return false;
    uint32_t save = c.i;
    if (c.ch() == '@') {
        Str g;
        Cur d = c;
        if (d.nonws(g) && d.ws1()) c = d;  // `@!?\S+\s+` (\S+ may include '!')
    }
    auto tail = [&](Cur e) -> bool {
        if (!e.lit("bra")) return false;
        Cur f = e;
        if (f.lit(".U") && f.ws1()) {
            if (f.word(tgt) && f.lit(";")) return true;
        }
        return e.ws1() && e.word(tgt) && e.lit(";");
    };
    if (tail(c)) return true;
    c.i = save;
    return tail(c);
}
// substring test
OCB_HD inline bool str_has(Str s, Str sub) {
    if (sub.n == 0) return true;
    for (uint32_t i = 0; i + sub.n <= s.n; ++i) {
        uint32_t j = 0;
        while (j < sub.n && s.p[i + j] == sub.p[j]) ++j;
        if (j == sub.n) return true;
    }
    return false;
}
// re.sub(escape(reg) + r'(?!\d)', to, line)
OCB_HD inline Str sub_reg(Arena &a, Str line, Str reg_, Str to, bool &changed) {
    changed = false;
    SB b;
    b.init(a, line.n + 8);
    uint32_t i = 0;
    while (i < line.n) {
        if (i + reg_.n <= line.n && mem_eq(line.p + i, reg_.p, reg_.n) &&
            !(i + reg_.n < line.n && is_dg(line.p[i + reg_.n]))) {
            b.s(to);
            i += reg_.n;
            changed = true;
        } else {
            b.c(line.p[i++]);
        }
    }
    return changed ? b.str() : line;
}
// every %rd<digits> number on a line
template <class F>
OCB_HD inline void each_rd(Str l, F fn) {
    for (uint32_t i = 0; i + 3 < l.n + 1; ++i) {
        if (l.p[i] == '%' && i + 2 < l.n && l.p[i + 1] == 'r' && l.p[i + 2] == 'd' && i + 3 < l.n &&
            is_dg(l.p[i + 3])) {
            uint32_t j = i + 3;
            int64_t v = 0;
            while (j < l.n && is_dg(l.p[j])) {
                v = v * 10 + (l.p[j] - '0');
                if (v > 100000000) v = 100000000;
                ++j;
            }
            fn(v);
            i = j - 1;
        }
    }
}

// The text peepholes of emit_kernel (emit.py:688-1021), in order.
OCB_HD inline void Emit::peepholes(Vec<Str> &L) {
    // (1) shl.b32 + cvt.s64.s32 -> cvt.u64.u32 + shl.b64
    for (uint32_t i = 0; i + 1 < L.n; ++i) {
        Str d, s, n, d2, s2;
        if (pat_shl(L[i], d, s, n) && pat_cvt64(L[i + 1], d2, s2) && eq(d, s2)) {
            SB a = sb();
            a.s("    cvt.u64.u32 ").s(d2).s(", ").s(s).c(';');
            SB b = sb();
            b.s("    shl.b64 ").s(d2).s(", ").s(d2).s(", ").s(n).c(';');
            L[i] = a.str();
            L[i + 1] = b.str();
        }
    }
    // (2) guard loads feeding a predicated-mov pair
    {
        struct Ins { uint32_t at; Str line; };
        Vec<Ins> ins;
        ins.init();
        uint32_t counter = 0;
        for (uint32_t i = 0; i + 2 < L.n; ++i) {
            Str ind, dst, gp, gs, np, nd, nv;
            if (!pat_ld(L[i], ind, dst)) continue;
            if (pat_pmov_reg(L[i + 1], gp, gs) && pat_nmov_any(L[i + 2], np, nd, nv) && eq(gp, np) && eq(gs, dst)) {
                SB lbl = sb();
                lbl.s("_ld_skip_").i(counter++);
                SB b = sb();
                b.s(ind).s("@!").s(gp).s(" bra ").s(lbl.str()).c(';');
                ins.push(tmp, Ins{i, b.str()});
                SB l2 = sb();
                l2.s(lbl.str()).c(':');
                ins.push(tmp, Ins{i + 1, l2.str()});
            }
        }
        if (ins.n) {
            Vec<Str> nl;
            nl.init();
            if (!nl.reserve(ar, L.n + ins.n)) return;
            // inserting in reverse order at the recorded indices == stable merge
            uint32_t q = 0;
            for (uint32_t i = 0; i <= L.n; ++i) {
                while (q < ins.n && ins[q].at == i) nl.push(ar, ins[q++].line);
                if (i < L.n) nl.push(ar, L[i]);
            }
            L = nl;
        }
    }
    // (3) @p mov + @!p mov -> selp
    {
        uint32_t i = 0;
        while (i + 1 < L.n) {
            Str ind, p1, ty, d1, sv, p2, d2, fv;
            if (pat_pmov(L[i], ind, p1, ty, d1, sv)) {
                Cur c{L[i + 1], 0};
                // `^(\s+)@!(%\w+)\s+mov\.(\w+)\s+(%\w+),\s*(\S+);$`
                Str t2;
                bool ok = c.ws1() && c.lit("@!") && c.reg(p2) && c.ws1() && c.lit("mov.") && c.word(t2) &&
                          c.ws1() && c.reg(d2) && c.lit(",");
                if (ok) {
                    c.ws0();
                    uint32_t st = c.i;
                    Str l1 = L[i + 1];
                    ok = l1.n >= st + 2 && l1.p[l1.n - 1] == ';';
                    for (uint32_t q = st; ok && q < l1.n; ++q) ok = !is_wsc(l1.p[q]);
                    if (ok) fv = Str{l1.p + st, l1.n - 1 - st};
                }
                if (ok && eq(p1, p2) && eq(d1, d2)) {
                    SB b = sb();
                    b.s(ind).s("selp.").s(ty).c(' ').s(d1).s(", ").s(sv).s(", ").s(fv).s(", ").s(p1).c(';');
                    L[i] = b.str();
                    L.erase(i + 1);
                    if (i + 1 < L.n) {
                        Str fd, fs;
                        if (pat_mov_full(L[i + 1], fd, fs) && eq(fs, d1)) {
                            SB b2 = sb();
                            b2.s(ind).s("selp.").s(ty).c(' ').s(fd).s(", ").s(sv).s(", ").s(fv).s(", ").s(p1).c(';');
                            L[i] = b2.str();
                            L.erase(i + 1);
                        }
                    }
                }
            }
            ++i;
        }
    }
    // (4) mov.bNN copy propagation.  Each line's destination register is
    // parsed once and kept aligned with L (a substitution never changes a
    // line's destination; an erase removes one entry), and label positions
    // are cached per branch target (an erased mov line is never a label, so
    // an erase only moves the labels after it up by one).
    {
        Vec<Str> dests;  // pat_dest of each line, n = 0 when the line has none
        dests.init();
        if (!dests.reserve(tmp, L.n + 1)) { unsup(); return; }
        for (uint32_t j = 0; j < L.n; ++j) {
            Str dd;
            dests.p[j] = pat_dest(L[j], dd) ? dd : Str{nullptr, 0};
        }
        dests.n = L.n;
        struct LabelPos { Str tgt; int64_t pos; };
        Vec<LabelPos> labels;
        labels.init();
        auto label_pos = [&](Str tgt) -> int64_t {
            for (uint32_t q = 0; q < labels.n; ++q)
                if (eq(labels[q].tgt, tgt)) return labels[q].pos;
            // the last "name:" line (not indented) with that name
            int64_t pos = -1;
            for (uint32_t q = 0; q < L.n; ++q) {
                Str ln = L[q];
                uint32_t e = ln.n;
                while (e && is_wsc(ln.p[e - 1])) --e;
                if (e && ln.p[e - 1] == ':' && !(ln.n && ln.p[0] == ' ') && e - 1 == tgt.n &&
                    mem_eq(ln.p, tgt.p, tgt.n))
                    pos = q;
            }
            labels.push(tmp, LabelPos{tgt, pos});
            return pos;
        };
        uint32_t i = 0;
        uint32_t guard = 0;
        while (i < L.n && !bad()) {
            if (++guard > 50000000u) { unsup(); return; }
            Str dst, src;
            if (pat_movb(L[i], dst, src) && eq(reg_class(dst), reg_class(src))) {
                int64_t src_redef = -1;
                for (uint32_t j = i + 1; j < L.n; ++j) {
                    Str dd = dests[j];
                    if (dd.n) {
                        if (eq(dd, dst)) break;
                        if (eq(dd, src)) {
                            src_redef = j;
                            break;
                        }
                    }
                }
                bool unsafe = false;
                if (src_redef >= 0) {
                    for (uint32_t j = (uint32_t)src_redef + 1; j < L.n; ++j) {
                        if (dests[j].n && eq(dests[j], dst)) break;
                        if (str_has(L[j], dst)) {
                            unsafe = true;
                            break;
                        }
                    }
                }
                if (!unsafe && src_redef >= 0) {
                    // any backward branch from line i on
                    for (uint32_t j = i; j < L.n && !unsafe; ++j) {
                        Str tgt;
                        if (!pat_bra(L[j], tgt)) continue;
                        int64_t pos = label_pos(tgt);
                        if (pos >= 0 && pos <= (int64_t)j) unsafe = true;
                    }
                }
                if (unsafe) {
                    ++i;
                    continue;
                }
                L.erase(i);
                dests.erase(i);
                for (uint32_t q = 0; q < labels.n; ++q)
                    if (labels[q].pos > (int64_t)i) labels[q].pos--;
                for (uint32_t j = i; j < L.n; ++j) {
                    Str dd = dests[j];
                    bool isd = dd.n != 0;
                    if (isd && eq(dd, dst)) break;
                    bool redef_src = isd && eq(dd, src);
                    bool ch;
                    L[j] = sub_reg(ar, L[j], dst, src, ch);
                    if (ch) {
                        Str nd;
                        dests.p[j] = pat_dest(L[j], nd) ? nd : Str{nullptr, 0};
                    }
                    if (redef_src) break;
                }
                continue;
            }
            ++i;
        }
    }
    // (5) rd compaction through in-place address adds
    rd_compact(L);
}

// The %rd compaction of the text peepholes (emit.py:556-614 for .func bodies,
// the same logic as the kernel entry's): when a cvt writes the highest %rd
// and two or more add.u64 read it, the adds write their pointer operand in
// place; then the highest register is renamed into each gap.  True when the
// rewrite ran.
OCB_HD inline bool Emit::rd_compact(Vec<Str> &L) {
    bool ran = false;
    {
        int64_t rd_max = -1;
        for (uint32_t i = 0; i < L.n; ++i) each_rd(L[i], [&](int64_t v) { if (v > rd_max) rd_max = v; });
        rd_max += 1;
        if (rd_max > 3) {
            SB hb = sb();
            hb.s("%rd").i(rd_max - 1);
            Str highest = hb.str();
            int64_t cvt_idx = -1;
            for (uint32_t i = 0; i < L.n && cvt_idx < 0; ++i) {
                Str l = L[i];
                if (!str_has(l, S("cvt")) || !str_has(l, highest)) continue;
                // l.strip().split()[1].rstrip(',') == highest
                uint32_t a = 0;
                while (a < l.n && is_wsc(l.p[a])) ++a;
                while (a < l.n && !is_wsc(l.p[a])) ++a;
                while (a < l.n && is_wsc(l.p[a])) ++a;
                uint32_t b = a;
                while (b < l.n && !is_wsc(l.p[b])) ++b;
                if (a == b) { unsup(); return false; }  // split()[1] raises IndexError
                Str tok{l.p + a, b - a};
                while (tok.n && tok.p[tok.n - 1] == ',') tok.n--;
                if (eq(tok, highest)) cvt_idx = i;
            }
            // add.u64 (%rd\d+),\s*(%rd\d+),\s*<highest>  (re.search)
            struct Add { uint32_t at; Str dst, ptr; };
            Vec<Add> adds;
            adds.init();
            for (uint32_t i = 0; i < L.n; ++i) {
                Str l = L[i];
                if (!str_has(l, S("add.u64")) || !str_has(l, highest)) continue;
                bool found = false;
                for (uint32_t s0 = 0; s0 + 7 <= l.n && !found; ++s0) {
                    Cur c{l, s0};
                    if (!c.lit("add.u64") || !c.ws1()) continue;
                    Str d, p;
                    auto rdreg = [&](Str &out) -> bool {
                        uint32_t st = c.i;
                        if (!c.lit("%rd")) return false;
                        Str dg;
                        if (!c.digits(dg)) { c.i = st; return false; }
                        out = Str{l.p + st, c.i - st};
                        return true;
                    };
                    if (!rdreg(d) || !c.lit(",")) continue;
                    c.ws0();
                    if (!rdreg(p) || !c.lit(",")) continue;
                    c.ws0();
                    if (!c.lit("")) continue;
                    Cur h = c;
                    bool hm = true;
                    for (uint32_t q = 0; q < highest.n; ++q, ++h.i)
                        if (h.i >= l.n || l.p[h.i] != highest.p[q]) { hm = false; break; }
                    if (!hm) continue;
                    adds.push(tmp, Add{i, d, p});
                    found = true;
                }
            }
            if (cvt_idx >= 0 && adds.n >= 2) {
                ran = true;
                for (int64_t q = (int64_t)adds.n - 1; q >= 0; --q) {
                    Add &A = adds[(uint32_t)q];
                    if (eq(A.dst, A.ptr)) continue;
                    // replace the first "add.u64 <dst>, <ptr>" with "add.u64 <ptr>, <ptr>"
                    SB from = sb();
                    from.s("add.u64 ").s(A.dst).s(", ").s(A.ptr);
                    Str fr = from.str();
                    Str l = L[A.at];
                    for (uint32_t s0 = 0; s0 + fr.n <= l.n; ++s0) {
                        if (mem_eq(l.p + s0, fr.p, fr.n)) {
                            SB nb = sb();
                            nb.s(Str{l.p, s0}).s("add.u64 ").s(A.ptr).s(", ").s(A.ptr).s(Str{l.p + s0 + fr.n, l.n - s0 - fr.n});
                            L[A.at] = nb.str();
                            break;
                        }
                    }
                    for (uint32_t i = A.at + 1; i < L.n; ++i) {
                        if (!str_has(L[i], A.dst)) continue;
                        bool ch;
                        L[i] = sub_reg(ar, L[i], A.dst, A.ptr, ch);
                    }
                }
                // compact: rename the top register into each gap
                int64_t top = -1;
                uint32_t cap = 0;
                for (uint32_t i = 0; i < L.n; ++i) each_rd(L[i], [&](int64_t v) { if (v > top) top = v; });
                if (top >= 0) {
                    cap = (uint32_t)top + 1;
                    uint8_t *used = (uint8_t *)tmp.alloc(cap + 1, 16);
                    if (!used) { unsup(); return false; }
                    for (uint32_t i = 0; i <= cap; ++i) used[i] = 0;
                    for (uint32_t i = 0; i < L.n; ++i) each_rd(L[i], [&](int64_t v) { used[v] = 1; });
                    int64_t cur_top = top;
                    for (uint32_t gap = 0; gap < cap; ++gap) {
                        if (used[gap]) continue;
                        // top = max(used_rds)
                        while (cur_top >= 0 && !used[cur_top]) --cur_top;
                        if (cur_top > (int64_t)gap) {
                            SB tf = sb();
                            tf.s("%rd").i(cur_top);
                            SB tt = sb();
                            tt.s("%rd").i(gap);
                            for (uint32_t i = 0; i < L.n; ++i) {
                                bool ch;
                                L[i] = sub_reg(ar, L[i], tf.str(), tt.str(), ch);
                            }
                            used[cur_top] = 0;
                            used[gap] = 1;
                        }
                    }
                }
            }
        }
    }
    return ran;
}

// ---- if_convert_diamonds gate (optimizer/if_convert.py:88-228) ------------------
// The rewrite fires only on load+mul+store diamonds whose condition compares a
// load of the parent block; a kernel where it would fire is declined.
OCB_HD inline bool if_convert_would_fire(Module &m, Kernel &k) {
    auto blk = [&](Str l) -> int32_t {
        int32_t r = -1;
        for (uint32_t i = 0; i < k.blocks.n; ++i)
            if (eq(m.blocks[k.blocks[i]].label, l)) r = (int32_t)k.blocks[i];
        return r;
    };
    auto arm = [&](int32_t b, Opnd &cst) -> bool {
        Block &B = m.blocks[(uint32_t)b];
        if (B.term.kind != T_BR) return false;
        int32_t st = -1, mu = -1, ld = -1;
        for (int32_t q = (int32_t)B.insts.n - 1; q >= 0; --q) {
            const Inst &in = m.insts[B.insts[q]];
            if (in.kind == I_STORE && st < 0) st = (int32_t)B.insts[q];
            else if (in.kind == I_BIN && in.op == BO_MUL && mu < 0) mu = (int32_t)B.insts[q];
            else if (in.kind == I_LOAD && ld < 0) ld = (int32_t)B.insts[q];
        }
        if (st < 0 || mu < 0 || ld < 0) return false;
        const Inst &S_ = m.insts[st], &M = m.insts[mu], &L = m.insts[ld];
        if (!(S_.b.k == O_VAL && m.vals[S_.b.x].id == m.vals[M.dest].id)) return false;
        uint32_t lid = m.vals[L.dest].id;
        if (M.a.k == O_VAL && m.vals[M.a.x].id == lid && M.b.k == O_CONST) cst = M.b;
        else if (M.b.k == O_VAL && m.vals[M.b.x].id == lid && M.a.k == O_CONST) cst = M.a;
        else return false;
        return true;
    };
    for (uint32_t i = 0; i < k.blocks.n; ++i) {
        Block &bb = m.blocks[k.blocks[i]];
        if (bb.term.kind != T_CBR) continue;
        int32_t tb = blk(bb.term.t), fb = blk(bb.term.f);
        if (tb < 0 || fb < 0) continue;
        Block &T = m.blocks[(uint32_t)tb], &F = m.blocks[(uint32_t)fb];
        if (T.term.kind != T_BR || F.term.kind != T_BR || !eq(T.term.t, F.term.t)) continue;
        Opnd tc, fc;
        if (!arm(tb, tc) || !arm(fb, fc)) continue;
        if (m.consts[tc.x].pyfloat != m.consts[fc.x].pyfloat) continue;
        int32_t pl = -1, cmp = -1;
        for (uint32_t q = 0; q < bb.insts.n; ++q) {
            const Inst &in = m.insts[bb.insts[q]];
            if (in.kind == I_CMP) cmp = (int32_t)bb.insts[q];
            if (in.kind == I_LOAD) pl = (int32_t)bb.insts[q];
        }
        if (pl < 0 || cmp < 0) continue;
        const Inst &C = m.insts[cmp];
        uint32_t lid = m.vals[m.insts[pl].dest].id;
        if ((C.a.k == O_VAL && m.vals[C.a.x].id == lid) || (C.b.k == O_VAL && m.vals[C.b.x].id == lid))
            return true;
    }
    return false;
}

// ---- emit_kernel (emit.py:648-1126) -------------------------------------------------
OCB_HD inline bool Emit::emit_kernel(Kernel &kk, Vec<Str> &out) {
    k = &kk;
    tmp.used = 0;
    nid0 = k->next_id;
    fb_alloc = nullptr;
    fb_cap = 0;
    widen = nullptr;
    widen_cap = 0;
    for (int p = 0; p < PF_N; ++p) fb_count[p] = reg_counts[p] = 0;
    skip.init(tmp, 2 * k->blocks.n + 8);
    term_depth = 0;
    lt_ok = false;
    // names must stay ASCII (the reference's \w is Unicode-aware)
    for (uint32_t i = 0; i < k->params.n; ++i)
        for (uint32_t q = 0; q < k->params[i].name.n; ++q)
            if ((uint8_t)k->params[i].name.p[q] >= 0x80) { unsup(); return false; }
    build_alloc();
    if (bad()) return false;
    // shared pointer values by declaration name (scan order)
    struct SVE { uint32_t s; uint32_t vx; };
    Vec<SVE> svals;
    svals.init();
    if (k->shared.n) {
        for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
            Block &b = B(k->blocks[bi]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = I(b.insts[ii]);
                Opnd cand[3];
                int nc = 0;
                if (in.kind == I_BIN || in.kind == I_CMP) cand[nc++] = in.a;    // .lhs
                if (in.dest >= 0) cand[nc++] = ov((uint32_t)in.dest);          // .dest
                if (in.kind == I_LOAD || in.kind == I_STORE) cand[nc++] = in.a; // .addr
                for (int q = 0; q < nc; ++q) {
                    if (cand[q].k != O_VAL) continue;
                    const Value &v = V(cand[q].x);
                    if (!is_ptr(v.ty)) continue;
                    for (uint32_t s = 0; s < k->shared.n; ++s)
                        if (eq(k->shared[s].name, v.name)) {
                            svals.push(tmp, SVE{s, cand[q].x});
                            break;
                        }
                }
            }
        }
    }
    // printf format strings of this kernel, in block order (emit.py:681-690)
    pfs.init();
    pf_idx = pf_count = 0;
    for (uint32_t bi = 0; bi < k->blocks.n; ++bi) {
        Block &b = B(k->blocks[bi]);
        for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
            const Inst &in = I(b.insts[ii]);
            if (in.kind != I_PRINTF) continue;
            SB lb = sb();
            lb.s("_fmt_").s(k->name).c('_').i(pfs.n);
            pfs.push(ar, PFmt{lb.str(), in.func});
        }
    }
    Vec<Str> body;
    body.init();
    lines = &body;
    for (uint32_t bi = 0; bi < k->blocks.n && !bad(); ++bi) emit_block(k->blocks[bi]);
    if (bad()) return false;
    peepholes(body);
    if (bad()) return false;
    // header
    out.push(ar, S(".version 9.0"));
    out.push(ar, S(".target sm_120"));
    out.push(ar, S(".address_size 64"));
    out.push(ar, S(""));
    SB pl = sb();
    {
        NameSet seen;
        seen.init();
        bool first = true;
        // struct parameters flatten to one .param per leaf field named
        // `<param>_<field>`; a name seen before is skipped (emit.py:975-989)
        struct Leaf {
            Str name;
            Ty ty;
            uint32_t f;    // next field to visit (struct frames)
        };
        Leaf stack[24];
        for (uint32_t i = 0; i < k->params.n; ++i) {
            uint32_t sp = 0;
            stack[sp++] = Leaf{k->params[i].name, k->params[i].ty, 0};
            while (sp) {
                Leaf &top = stack[sp - 1];
                if (ty_is_struct(top.ty)) {
                    if (top.f >= m.nfields(top.ty)) {
                        --sp;
                        continue;
                    }
                    const SField &fd = m.field(top.ty, top.f++);
                    if (sp >= 24) { unsup(); return false; }
                    Str nm = cat(tmp, top.name, S("_"), fd.name);
                    stack[sp++] = Leaf{nm, fd.ty, 0};
                    continue;
                }
                Str pn = top.name;
                Ty pty = top.ty;
                --sp;
                if (seen.has(pn)) continue;
                seen.add(tmp, pn);
                const char *t = ptx_type(pty);
                if (cstr_eq(t, "f16")) t = "b16";
                if (!first) pl.s(", ");
                first = false;
                pl.s(".param .").s(t).c(' ').s(pn);
            }
        }
    }
    SB ve = sb();
    ve.s(".visible .entry ").s(k->name).c('(');
    out.push(ar, ve.str());
    SB pv = sb();
    pv.s("    ").s(pl.str()).c(')');
    out.push(ar, pv.str());
    if (k->n_launch) {
        SB b = sb();
        b.s(".maxntid ").i(k->launch[0]).s(", 1, 1");
        out.push(ar, b.str());
        if (k->n_launch > 1) {
            SB b2 = sb();
            b2.s(".minnctapersm ").i(k->launch[1]);
            out.push(ar, b2.str());
        }
    }
    out.push(ar, S("{"));
    for (uint32_t s = 0; s < k->shared.n; ++s) {
        const SharedDecl &d = k->shared[s];
        if (d.count == 0) {
            SB b = sb();
            uint32_t al = ty_is_scalar(d.ty) ? ty_size(d.ty) : 4;
            b.s(".extern .shared .align ").i(al).s(" .b8 ").s(d.name).s("[];");
            bool dup = false;
            for (uint32_t q = 0; q < preamble.n && !dup; ++q) dup = eq(preamble[q], b.str());
            if (!dup) preamble.push(ar, b.str());
        } else {
            SB b = sb();
            if (ty_is_struct(d.ty))  // raw bytes with the fields' alignment
                b.s("    .shared .align ").i(m.struct_align(d.ty)).s(" .b8 ").s(d.name).c('[')
                    .i((pyint)m.tsize(d.ty) * d.count).s("];");
            else
                b.s("    .shared .").s(ptx_type(d.ty)).c(' ').s(d.name).c('[').i(d.count).s("];");
            out.push(ar, b.str());
        }
    }
    for (uint32_t q = 0; q < k->locals.n; ++q) {
        const LocalDecl &d = k->locals[q];
        int64_t eb = m.tsize(d.ty);
        int64_t al = 1;
        while (al < eb) al <<= 1;
        if (al > 16) al = 16;
        SB b = sb();
        b.s("    .local .align ").i(al).s(" .b8 _local_").i(V(d.val).id).c('[').i(eb * d.count).s("];");
        out.push(ar, b.str());
    }
    // register counts from the text (prefixes rd, fd, r, f, h, p; longest first)
    int cnt[PF_N];
    bool any = false;
    for (int p = 0; p < PF_N; ++p) cnt[p] = 0;
    for (uint32_t i = 0; i < body.n; ++i) {
        Str l = body[i];
        for (uint32_t j = 0; j + 1 < l.n; ++j) {
            if (l.p[j] != '%') continue;
            uint32_t a = j + 1;
            int pf = -1;
            if (a + 1 < l.n && l.p[a] == 'r' && l.p[a + 1] == 'd') { pf = PF_RD; a += 2; }
            else if (a + 1 < l.n && l.p[a] == 'f' && l.p[a + 1] == 'd') { pf = PF_FD; a += 2; }
            else if (l.p[a] == 'r') { pf = PF_R; a += 1; }
            else if (l.p[a] == 'f') { pf = PF_F; a += 1; }
            else if (l.p[a] == 'h') { pf = PF_H; a += 1; }
            else if (l.p[a] == 'p') { pf = PF_P; a += 1; }
            if (pf < 0 || a >= l.n || !is_dg(l.p[a])) {
                // the alternation backtracks: %rd<non-digit> may still match as %r? no: 'rd'
                // fails and 'r' needs a digit next, which 'd' is not; likewise for 'fd'.
                continue;
            }
            int64_t v = 0;
            while (a < l.n && is_dg(l.p[a])) {
                v = v * 10 + (l.p[a] - '0');
                if (v > 100000000) v = 100000000;
                ++a;
            }
            if (cnt[pf] < v + 1) cnt[pf] = (int)(v + 1);
            any = true;
            j = a - 1;
        }
    }
    if (any)
        for (int p = 0; p < PF_N; ++p) reg_counts[p] = cnt[p];
    // declarations sorted by prefix name: f, fd, h, p, r, rd
    int order[] = {PF_F, PF_FD, PF_H, PF_P, PF_R, PF_RD};
    for (int oi = 0; oi < PF_N; ++oi) {
        int p = order[oi];
        bool present = any ? cnt[p] > 0 : reg_counts[p] > 0;
        if (!present || p == PF_P) continue;
        SB b = sb();
        const char *t = p == PF_RD ? ".b64" : p == PF_F ? ".f32" : p == PF_FD ? ".f64" : p == PF_H ? ".f16" : ".b32";
        b.s("    .reg ").s(t).s(" %").s(pf_name(p)).c('<').i(reg_counts[p]).s(">;");
        out.push(ar, b.str());
    }
    {
        int pc = reg_counts[PF_P] > 1 ? reg_counts[PF_P] : 1;
        bool has_p = any ? cnt[PF_P] > 0 : reg_counts[PF_P] > 0;
        if (!has_p) pc = 1;
        SB b = sb();
        b.s("    .reg .pred %p<").i(pc).s(">;");
        out.push(ar, b.str());
    }
    out.push(ar, S(""));
    // initialisers: shared bases first, then local bases, then the body
    lines = &out;
    {
        Vec<Str> seen;
        seen.init();
        for (uint32_t s = 0; s < k->shared.n; ++s)
            for (uint32_t q = 0; q < svals.n; ++q) {
                if (svals[q].s != s) continue;
                Str r = reg(svals[q].vx);
                bool dup = false;
                for (uint32_t z = 0; z < seen.n && !dup; ++z) dup = eq(seen[z], r);
                if (dup) continue;
                seen.push(tmp, r);
                SB b = sb();
                b.s("    mov.u64 ").s(r).s(", ").s(k->shared[s].name).c(';');
                out.push(ar, b.str());
            }
        seen.init();
        for (uint32_t q = 0; q < k->locals.n; ++q) {
            Str r = reg(k->locals[q].val);
            bool dup = false;
            for (uint32_t z = 0; z < seen.n && !dup; ++z) dup = eq(seen[z], r);
            if (dup) continue;
            seen.push(tmp, r);
            SB b = sb();
            b.s("    mov.u64 ").s(r).s(", _local_").i(V(k->locals[q].val).id).c(';');
            out.push(ar, b.str());
        }
    }
    for (uint32_t i = 0; i < body.n; ++i) out.push(ar, body[i]);
    out.push(ar, S("}"));
    // the vprintf declaration (once per module) and this kernel's format
    // strings as byte arrays join the module preamble (emit.py:1110-1125)
    if (pfs.n) {
        if (!vprintf_decl) {
            vprintf_decl = true;
            preamble.push(ar, S(".extern .func (.param .b32 func_retval0) vprintf(.param .b64 fmt, "
                                ".param .b64 valist);"));
            preamble.push(ar, S(""));
        }
        for (uint32_t q = 0; q < pfs.n; ++q) {
            bool dup = false;
            for (uint32_t z = 0; z < fmt_done.n && !dup; ++z) dup = eq(fmt_done[z], pfs[q].label);
            if (dup) continue;
            fmt_done.push(ar, pfs[q].label);
            Str f = pfs[q].fmt;
            SB b = sb();
            b.s(".global .align 1 .b8 ").s(pfs[q].label).c('[').i((pyint)f.n + 1).s("] = {");
            for (uint32_t z = 0; z < f.n; ++z) b.i((uint8_t)f.p[z]).s(", ");
            b.s("0};");
            preamble.push(ar, b.str());
        }
    }
    return !bad();
}

// `.param .<type> <name>` list of a device function (f16 spelled b16)
OCB_HD inline Str devfn_params(Emit &E, const Kernel &f) {
    SB b = E.sb();
    for (uint32_t i = 0; i < f.params.n; ++i) {
        const char *t = ptx_type(f.params[i].ty);
        if (cstr_eq(t, "f16")) t = "b16";
        if (i) b.s(", ");
        b.s(".param .").s(t).c(' ').s(f.params[i].name);
    }
    return b.str();
}
// `.func [(.param .<ret> retval0) ]__devfn_<name>(`
OCB_HD inline void devfn_head(SB &b, const Kernel &f) {
    b.s(".func ");
    if (!(ty_is_scalar(f.ret) && ty_scalar(f.ret) == S_VOID)) {
        const char *t = ptx_type(f.ret);
        if (cstr_eq(t, "f16")) t = "b16";
        b.s("(.param .").s(t).s(" retval0) ");
    }
    b.s("__devfn_").s(f.name).c('(');
}

// ---- emit_device_function (emit.py:506-646) --------------------------------------
// The body as in a kernel but without the kernel's text peepholes (only the
// %rd compaction), registers declared from the text in prefix order, locals
// by their variable names.  The fallback registers of emission-time values
// count from zero: the reference keeps the allocation counts of the previous
// kernel there, and device functions are emitted before any kernel.
OCB_HD inline bool Emit::emit_devfn(Kernel &kk, Vec<Str> &out) {
    k = &kk;
    tmp.used = 0;
    nid0 = k->next_id;
    fb_alloc = nullptr;
    fb_cap = 0;
    widen = nullptr;
    widen_cap = 0;
    for (int p = 0; p < PF_N; ++p) fb_count[p] = reg_counts[p] = 0;
    skip.init(tmp, 2 * k->blocks.n + 8);
    term_depth = 0;
    lt_ok = false;
    pfs.init();
    pf_idx = pf_count = 0;
    for (uint32_t i = 0; i < k->params.n; ++i)
        for (uint32_t q = 0; q < k->params[i].name.n; ++q)
            if ((uint8_t)k->params[i].name.p[q] >= 0x80) { unsup(); return false; }
    build_alloc();
    if (bad()) return false;
    for (int p = 0; p < PF_N; ++p) alloc_max[p] = 0;
    Vec<Str> body;
    body.init();
    lines = &body;
    for (uint32_t bi = 0; bi < k->blocks.n && !bad(); ++bi) emit_block(k->blocks[bi]);
    if (bad()) return false;
    // %(\w+?)(\d+) over the body: the count per register prefix
    int cnt[PF_N];
    bool any = false;
    for (int p = 0; p < PF_N; ++p) cnt[p] = 0;
    for (uint32_t i = 0; i < body.n; ++i) {
        Str l = body[i];
        for (uint32_t j = 0; j < l.n; ++j) {
            if (l.p[j] != '%') continue;
            uint32_t a = j + 1, e = a;
            auto wch = [](char c) {
                return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '_';
            };
            while (e < l.n && wch(l.p[e])) ++e;
            // the shortest \w+ prefix followed by digits (then as many digits as follow)
            uint32_t ps = a + 1;
            bool hit = false;
            for (; ps < e; ++ps)
                if (l.p[ps] >= '0' && l.p[ps] <= '9') { hit = true; break; }
            if (!hit) { j = e > j ? e - 1 : j; continue; }
            uint32_t de = ps;
            while (de < l.n && l.p[de] >= '0' && l.p[de] <= '9') ++de;
            Str pre{l.p + a, ps - a};
            int pf = eq(pre, "rd") ? PF_RD : eq(pre, "fd") ? PF_FD : eq(pre, "r") ? PF_R :
                     eq(pre, "f") ? PF_F : eq(pre, "h") ? PF_H : eq(pre, "p") ? PF_P : -1;
            if (pf >= 0) {
                int64_t v = 0;
                for (uint32_t q = ps; q < de && v < 100000000; ++q) v = v * 10 + (l.p[q] - '0');
                if (cnt[pf] < v + 1) cnt[pf] = (int)(v + 1);
                any = true;
            }
            j = de - 1;
        }
    }
    bool any_rd_prefix = any;
    if (cnt[PF_RD] > 3 && rd_compact(body)) {
        int64_t top = -1;
        for (uint32_t i = 0; i < body.n; ++i) each_rd(body[i], [&](int64_t v) { if (v > top) top = v; });
        cnt[PF_RD] = (int)(top + 1);
    }
    if (bad()) return false;
    (void)any_rd_prefix;
    SB hb = sb();
    devfn_head(hb, *k);
    out.push(ar, hb.str());
    SB pb = sb();
    pb.s("    ").s(devfn_params(*this, *k)).c(')');
    out.push(ar, pb.str());
    out.push(ar, S("{"));
    // sorted prefix names: f, fd, h, p, r, rd
    int order[] = {PF_F, PF_FD, PF_H, PF_P, PF_R, PF_RD};
    for (int oi = 0; oi < PF_N; ++oi) {
        int p = order[oi];
        int c = any ? cnt[p] : reg_counts[p];
        bool present = any ? cnt[p] > 0 : reg_counts[p] > 0;
        if (!present) continue;
        SB b = sb();
        const char *t = p == PF_P ? ".pred" : p == PF_H ? ".f16" : p == PF_F ? ".f32" :
                        p == PF_FD ? ".f64" : p == PF_RD ? ".b64" : ".b32";
        b.s("    .reg ").s(t).s(" %").s(pf_name(p)).c('<').i(c).s(">;");
        out.push(ar, b.str());
    }
    for (uint32_t q = 0; q < k->locals.n; ++q) {
        const LocalDecl &d = k->locals[q];
        int64_t es = ty_is_scalar(d.ty) ? (int64_t)ty_size(d.ty) : 8;
        int64_t al = es < 16 ? es : 16;
        SB b = sb();
        b.s("    .local .align ").i(al).s(" .b8 ").s(d.name).c('[').i(es * d.count).s("];");
        out.push(ar, b.str());
    }
    out.push(ar, S(""));
    for (uint32_t i = 0; i < body.n; ++i) out.push(ar, body[i]);
    out.push(ar, S("}"));
    out.push(ar, S(""));
    return !bad();
}

// ---- module text: ir_to_ptx + the CLI's --emit-ptx assembly ----------------------
OCB_HD inline bool emit_module(Module &m, Arena &tmp, Out &o, const char *arch) {
    Emit E(m, tmp);
    for (uint32_t ki = 0; ki < m.kernels.n; ++ki)
        if (if_convert_would_fire(m, m.kernels[ki])) {
            m.unsup = true;
            return false;
        }
    // recursive device functions: forward declarations, then definitions,
    // lead the module preamble (emit.py:3136-3154)
    for (uint32_t fi = 0; fi < m.funcs.n; ++fi) {
        SB b = E.sb();
        devfn_head(b, m.funcs[fi]);
        b.s(devfn_params(E, m.funcs[fi])).s(");");
        E.preamble.push(*m.ar, b.str());
    }
    for (uint32_t fi = 0; fi < m.funcs.n; ++fi) {
        Vec<Str> lines;
        lines.init();
        if (!E.emit_devfn(m.funcs[fi], lines)) return false;
        // the definition is one preamble entry: its lines joined by newlines
        SB b = E.sb();
        for (uint32_t q = 0; q < lines.n; ++q) {
            if (q) b.c('\n');
            b.s(lines[q]);
        }
        E.preamble.push(*m.ar, b.str());
    }
    // kernel texts, keyed by name in dict order (a later kernel with the same
    // name replaces the earlier text but keeps its position)
    struct KT { Str name; Vec<Str> lines; };
    Vec<KT> kts;
    kts.init();
    for (uint32_t ki = 0; ki < m.kernels.n; ++ki) {
        Vec<Str> lines;
        lines.init();
        if (!E.emit_kernel(m.kernels[ki], lines)) return false;
        bool placed = false;
        for (uint32_t q = 0; q < kts.n && !placed; ++q)
            if (eq(kts[q].name, m.kernels[ki].name)) {
                kts[q].lines = lines;
                placed = true;
            }
        if (!placed) kts.push(*m.ar, KT{m.kernels[ki].name, lines});
    }
    auto line = [&](Str s) {
        o.put(s);
        o.put('\n');
    };
    line(S(".version 9.0"));
    o.put(".target ");
    o.put(arch);
    o.put('\n');
    line(S(".address_size 64"));
    // module-level variable declarations lead the preamble (emit.py:3164-3190)
    if (m.gvars.n) {
        Vec<Str> pre;
        pre.init();
        for (uint32_t q = 0; q < m.gvars.n; ++q) {
            const GVar &g = m.gvars[q];
            SB b = E.sb();
            b.s(".visible .").s(g.space == AS_CONST ? "const" : "global").s(" .align ");
            if (ty_is_struct(g.elem)) {  // raw bytes for the whole struct (x count)
                b.i(m.struct_align(g.elem)).s(" .b8 ").s(g.name).c('[')
                    .i((pyint)m.tsize(g.elem) * g.count).s("];");
            } else {
                b.i(is_ptr(g.elem) ? 8 : (pyint)ty_size(g.elem)).s(" .").s(ptx_type(g.elem)).c(' ').s(g.name);
                if (g.count > 1) b.c('[').i(g.count).c(']');
                b.c(';');
            }
            pre.push(*m.ar, b.str());
        }
        for (uint32_t q = 0; q < E.preamble.n; ++q) pre.push(*m.ar, E.preamble[q]);
        E.preamble = pre;
    }
    // all lines are joined by '\n' without a trailing newline
    Vec<Str> all;
    all.init();
    all.push(*m.ar, S(""));
    if (E.preamble.n) {
        for (uint32_t q = 0; q < E.preamble.n; ++q) all.push(*m.ar, E.preamble[q]);
        all.push(*m.ar, S(""));
    }
    for (uint32_t q = 0; q < kts.n; ++q) {
        if (starts(kts[q].name, "__")) continue;
        Vec<Str> &L = kts[q].lines;
        uint32_t st = 0;
        for (uint32_t j = 0; j < L.n; ++j)
            if (starts(L[j], ".visible") || starts(L[j], "{")) {
                st = j;
                break;
            }
        for (uint32_t j = st; j < L.n; ++j) all.push(*m.ar, L[j]);
        all.push(*m.ar, S(""));
    }
    for (uint32_t q = 0; q < all.n; ++q) {
        if (q) o.put('\n');
        o.put(all[q]);
    }
    return !E.bad() && !o.full;
}

}  // namespace cc
}  // namespace ocb
