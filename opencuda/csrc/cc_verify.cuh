// IR verifier: restates opencuda/ir/verify_ir.py:86-316 (verify_kernel /
// verify_module) with the dominator sets of opencuda/ir/dominator.py:44-112,
// over the IR of one TU (after parse, or after optimize).
//
// Output (the oracle's text form of verify_module's dict): for every kernel
// with violations, in module order, a line `kernel <name>` followed by one
// line per error string, in the reference's order and wording.
//
// Labels: the reference keys its maps by label, so a label that several
// blocks share has the successors of its LAST block (label_to_bb), and
// predecessor lists collect edges from every block.  Dominator sets are
// bit vectors over the distinct labels, iterated in block-list order to the
// fixed point of the same equations (only reachable predecessors intersect;
// an unreachable label dominates only itself).
//
// The non-natural-loop check walks a Python set of body labels, whose order
// is not reproducible here: a back edge with two or more violations makes
// the TU unsupported.
#pragma once
#include "cc_opt_base.cuh"
#include "cc_dump.cuh"

namespace ocb {
namespace cc {

struct Verifier {
    Module &m;
    Arena &tmp;
    Out &o;
    bool unsup = false;

    OCB_HD Verifier(Module &mod, Arena &t, Out &out) : m(mod), tmp(t), o(out) {}

    OCB_HD static const char *class_name(uint8_t kind) {
        switch (kind) {
        case I_BIN: return "BinInst";
        case I_CMP: return "CmpInst";
        case I_SELECT: return "SelectInst";
        case I_LOAD: return "LoadInst";
        case I_STORE: return "StoreInst";
        case I_CVT: return "CvtInst";
        case I_CALL: return "CallInst";
        case I_PARAM: return "ParamInst";
        case I_PRINTF: return "PrintfInst";
        case I_ASM: return "AsmInst";
        default: return "GlobalAddrInst";
        }
    }

    // Value operands in _operand_values order: lhs, rhs, src, addr, value,
    // then args (SelectInst's operands are not among those attributes).
    template <class F>
    OCB_HD void each_use(const Inst &in, F f) {
        switch (in.kind) {
        case I_BIN:
        case I_CMP:
        case I_STORE:
            if (in.a.k == O_VAL) f(in.a.x);
            if (in.b.k == O_VAL) f(in.b.x);
            break;
        case I_CVT:
        case I_LOAD:
            if (in.a.k == O_VAL) f(in.a.x);
            break;
        default: break;
        }
        if (in.kind == I_ASM) return;  // AsmInst has no operand attribute read here
        for (uint32_t q = 0; q < in.args.n; ++q)
            if (in.args[q].k == O_VAL) f(in.args[q].x);
    }

    OCB_HD void put_repr(Str s) {  // repr() of a label (identifier text)
        o.put('\'');
        o.put(s);
        o.put('\'');
    }

    OCB_HD bool kernel(Kernel &k, bool check_reach) {
        const uint32_t nb = k.blocks.n;
        if (!nb) return true;
        // distinct labels, in first-seen order; lab[i] = label id of block i
        uint32_t *lab = (uint32_t *)tmp.alloc(4ull * nb, 16);
        Str *names = (Str *)tmp.alloc(sizeof(Str) * (uint64_t)nb, 16);
        int32_t *last_bb = (int32_t *)tmp.alloc(4ull * nb, 16);
        if (!lab || !names || !last_bb) return false;
        LabelMap lm;
        lm.build(tmp, m, k.blocks);  // label -> last block index with it
        uint32_t nl = 0;
        // label id = ordinal of first occurrence, indexed by the label's last block
        int32_t *first = (int32_t *)tmp.alloc(4ull * (m.blocks.n + 1), 16);
        if (!first) return false;
        {
            for (uint32_t i = 0; i < nb; ++i) {
                int32_t lb = lm.get(B(k.blocks[i]).label);
                first[lb] = -1;
            }
            for (uint32_t i = 0; i < nb; ++i) {
                int32_t lb = lm.get(B(k.blocks[i]).label);
                if (first[lb] < 0) {
                    first[lb] = (int32_t)nl;
                    names[nl] = B(k.blocks[i]).label;
                    last_bb[nl] = lb;
                    ++nl;
                }
                lab[i] = (uint32_t)first[lb];
            }
        }
        auto label_id = [&](Str l) -> int32_t {  // -1: no block has it
            int32_t b = lm.get(l);
            return b < 0 ? -1 : first[b];
        };
        // successors of each label (its last block), as label ids (-1: undefined)
        int32_t *succ = (int32_t *)tmp.alloc(8ull * nl, 16);
        if (!succ) return false;
        auto succ_of_block = [&](const Block &b, int32_t out[2]) -> int {
            int n = 0;
            if (b.term.kind == T_BR) out[n++] = label_id(b.term.t);
            else if (b.term.kind == T_CBR) {
                out[n++] = label_id(b.term.t);
                out[n++] = label_id(b.term.f);
            }
            return n;
        };
        uint8_t *nsucc = (uint8_t *)tmp.alloc(nl, 16);
        if (!nsucc) return false;
        for (uint32_t l = 0; l < nl; ++l) {
            int32_t s2[2];
            nsucc[l] = (uint8_t)succ_of_block(B((uint32_t)last_bb[l]), s2);
            succ[2 * l] = s2[0];
            succ[2 * l + 1] = s2[1];
        }

        // Check 1: terminator presence, branch targets
        auto head = [&](Str lbl) {
            o.put('[');
            o.put(k.name);
            o.put(':');
            o.put(lbl);
            o.put("] ");
        };
        uint64_t mark0 = o.n;
        o.put("kernel ");
        o.put(k.name);
        o.put('\n');
        uint64_t mark1 = o.n;
        for (uint32_t i = 0; i < nb; ++i) {
            const Block &b = B(k.blocks[i]);
            if (b.term.kind == T_NONE) {
                head(b.label);
                o.put("missing terminator\n");
                continue;
            }
            Str tg[2];
            int nt = 0;
            if (b.term.kind == T_BR) tg[nt++] = b.term.t;
            else if (b.term.kind == T_CBR) { tg[nt++] = b.term.t; tg[nt++] = b.term.f; }
            for (int q = 0; q < nt; ++q)
                if (label_id(tg[q]) < 0) {
                    head(b.label);
                    o.put("branch to undefined block ");
                    put_repr(tg[q]);
                    o.put('\n');
                }
        }
        // Check 2: reachability from the entry (the first block's label)
        uint8_t *reach = (uint8_t *)tmp.alloc(nl, 16);
        // work stack: every push follows an edge (at most 2 per block) or is
        // a DFS visit (once per label)
        const uint64_t stk_cap = 2ull * nb + 2ull * nl + 8;
        uint32_t *stk = (uint32_t *)tmp.alloc(4ull * stk_cap, 16);
        if (!reach || !stk) return false;
        for (uint32_t l = 0; l < nl; ++l) reach[l] = 0;
        {
            uint32_t sp = 0;
            stk[sp++] = lab[0];
            while (sp) {
                uint32_t l = stk[--sp];
                if (reach[l]) continue;
                reach[l] = 1;
                for (uint32_t q = 0; q < nsucc[l]; ++q) {
                    int32_t s = succ[2 * l + q];
                    if (s >= 0 && !reach[s] && sp < stk_cap) stk[sp++] = (uint32_t)s;
                }
            }
        }
        if (check_reach)
            for (uint32_t i = 0; i < nb; ++i)
                if (!reach[lab[i]]) {
                    head(B(k.blocks[i]).label);
                    o.put("block is unreachable from entry\n");
                }
        // Check 3: def map (first defining block's label id, def count)
        uint32_t nid = k.next_id;
        IdArr<uint32_t> dblock, dcount;
        dblock.init(tmp, nid, 0xFFFFFFFFu);
        dcount.init(tmp, nid, 0);
        if (tmp.oom) return false;
        for (uint32_t i = 0; i < nb; ++i) {
            const Block &b = B(k.blocks[i]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = m.insts[b.insts[ii]];
                if (in.kind == I_ASM) {  // the outputs are defined here
                    for (uint32_t q = 0; q < in.pidx; ++q) {
                        if (in.args[q].k != O_VAL) continue;
                        uint32_t id = m.vals[in.args[q].x].id;
                        if (id >= nid) return false;
                        dcount.set(id, dcount.get(id) + 1);
                        if (dblock.get(id) == 0xFFFFFFFFu) dblock.set(id, lab[i]);
                    }
                    continue;
                }
                if (in.dest < 0) continue;
                uint32_t id = m.vals[(uint32_t)in.dest].id;
                if (id >= nid) return false;
                dcount.set(id, dcount.get(id) + 1);
                if (dblock.get(id) == 0xFFFFFFFFu) dblock.set(id, lab[i]);
            }
        }
        auto is_smem = [&](uint32_t v) {
            Ty t = m.vals[v].ty;
            return is_ptr(t) && (ty_as(t) == AS_SHARED || ty_as(t) == AS_LOCAL);
        };
        auto undefined = [&](uint32_t v) {
            uint32_t id = m.vals[v].id;
            return id >= nid || dblock.get(id) == 0xFFFFFFFFu;
        };
        // Check 4: every use has a definition
        for (uint32_t i = 0; i < nb; ++i) {
            const Block &b = B(k.blocks[i]);
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = m.insts[b.insts[ii]];
                each_use(in, [&](uint32_t v) {
                    if (undefined(v) && !is_smem(v)) {
                        head(b.label);
                        o.put("use of undefined value %");
                        o.put(m.vals[v].name);
                        o.put(" (id=");
                        o.put_i64(m.vals[v].id);
                        o.put(") in ");
                        o.put(class_name(in.kind));
                        o.put('\n');
                    }
                });
            }
            if (b.term.kind == T_CBR && b.term.v.k == O_VAL && undefined(b.term.v.x)) {
                head(b.label);
                o.put("CondBrTerm uses undefined value %");
                o.put(m.vals[b.term.v.x].name);
                o.put(" (id=");
                o.put_i64(m.vals[b.term.v.x].id);
                o.put(")\n");
            }
        }
        // dominator sets: bit vectors of nl bits per label
        uint32_t W = (nl + 63) / 64;
        uint64_t *dom = (uint64_t *)tmp.alloc(8ull * W * nl, 16);
        uint64_t *nd = (uint64_t *)tmp.alloc(8ull * W, 16);
        // predecessor label lists (CSR), from every block's successors
        uint32_t *pcnt = (uint32_t *)tmp.alloc(4ull * (nl + 1), 16);
        if (!dom || !nd || !pcnt) return false;
        for (uint32_t l = 0; l <= nl; ++l) pcnt[l] = 0;
        uint32_t ne = 0;
        for (uint32_t i = 0; i < nb; ++i) {
            int32_t s2[2];
            int n = succ_of_block(B(k.blocks[i]), s2);
            for (int q = 0; q < n; ++q)
                if (s2[q] >= 0) { pcnt[s2[q] + 1]++; ne++; }
        }
        for (uint32_t l = 0; l < nl; ++l) pcnt[l + 1] += pcnt[l];
        uint32_t *pred = (uint32_t *)tmp.alloc(4ull * (ne + 1), 16);
        uint32_t *pfill = (uint32_t *)tmp.alloc(4ull * (nl + 1), 16);
        if (!pred || !pfill) return false;
        for (uint32_t l = 0; l < nl; ++l) pfill[l] = pcnt[l];
        for (uint32_t i = 0; i < nb; ++i) {
            int32_t s2[2];
            int n = succ_of_block(B(k.blocks[i]), s2);
            for (int q = 0; q < n; ++q)
                if (s2[q] >= 0) pred[pfill[s2[q]]++] = lab[i];
        }
        const uint32_t entry = lab[0];
        for (uint32_t l = 0; l < nl; ++l)
            for (uint32_t w = 0; w < W; ++w) {
                uint64_t full = (w + 1) * 64 <= nl ? ~0ull : ((1ull << (nl - w * 64)) - 1);
                dom[l * W + w] = l == entry ? 0 : full;
            }
        dom[entry * W + entry / 64] |= 1ull << (entry % 64);
        for (bool changed = true; changed;) {
            changed = false;
            for (uint32_t i = 0; i < nb; ++i) {
                uint32_t l = lab[i];
                if (l == entry) continue;
                bool any = false;
                for (uint32_t q = pcnt[l]; q < pcnt[l + 1]; ++q) {
                    uint32_t p = pred[q];
                    if (!reach[p]) continue;
                    for (uint32_t w = 0; w < W; ++w)
                        nd[w] = any ? (nd[w] & dom[p * W + w]) : dom[p * W + w];
                    any = true;
                }
                if (!any)
                    for (uint32_t w = 0; w < W; ++w) nd[w] = 0;
                nd[l / 64] |= 1ull << (l % 64);
                for (uint32_t w = 0; w < W; ++w)
                    if (nd[w] != dom[l * W + w]) {
                        dom[l * W + w] = nd[w];
                        changed = true;
                    }
            }
        }
        auto dominates = [&](uint32_t a, uint32_t b) {
            return a == b || ((dom[b * W + a / 64] >> (a % 64)) & 1ull);
        };
        // Check 5: single-definition values: the def block dominates the use
        for (uint32_t i = 0; i < nb; ++i) {
            const Block &b = B(k.blocks[i]);
            uint32_t ul = lab[i];
            if (!reach[ul]) continue;
            for (uint32_t ii = 0; ii < b.insts.n; ++ii) {
                const Inst &in = m.insts[b.insts[ii]];
                each_use(in, [&](uint32_t v) {
                    if (undefined(v)) return;
                    uint32_t id = m.vals[v].id;
                    if (dcount.get(id) != 1) return;
                    uint32_t dl = dblock.get(id);
                    if (dl == ul || dominates(dl, ul) || dominates(ul, dl)) return;
                    o.put('[');
                    o.put(k.name);
                    o.put("] dominance violation: %");
                    o.put(m.vals[v].name);
                    o.put(" (id=");
                    o.put_i64(id);
                    o.put(") defined in ");
                    put_repr(names[dl]);
                    o.put(" does not dominate use in ");
                    put_repr(b.label);
                    o.put('\n');
                });
            }
            if (b.term.kind == T_CBR && b.term.v.k == O_VAL && !undefined(b.term.v.x)) {
                uint32_t id = m.vals[b.term.v.x].id;
                uint32_t dl = dblock.get(id);
                if (dcount.get(id) == 1 && dl != ul && !dominates(dl, ul) && !dominates(ul, dl)) {
                    o.put('[');
                    o.put(k.name);
                    o.put("] dominance violation in CondBrTerm: %");
                    o.put(m.vals[b.term.v.x].name);
                    o.put(" (id=");
                    o.put_i64(id);
                    o.put(") defined in ");
                    put_repr(names[dl]);
                    o.put(" does not dominate use in ");
                    put_repr(b.label);
                    o.put('\n');
                }
            }
        }
        // Check 6: natural loops.  Back edges by an iterative DFS from the
        // entry that visits successors in order (the recursive _dfs2).
        uint8_t *state = (uint8_t *)tmp.alloc(nl, 16);  // 0 new, 1 on stack, 2 done
        uint32_t *it = (uint32_t *)tmp.alloc(4ull * nl, 16);
        uint32_t *be = (uint32_t *)tmp.alloc(8ull * (nl * 2 + 1), 16);
        if (!state || !it || !be) return false;
        for (uint32_t l = 0; l < nl; ++l) { state[l] = 0; it[l] = 0; }
        uint32_t nbe = 0, sp = 0;
        stk[sp++] = entry;
        state[entry] = 1;
        while (sp) {
            uint32_t l = stk[sp - 1];
            if (it[l] < nsucc[l]) {
                int32_t s = succ[2 * l + it[l]++];
                if (s < 0) continue;
                if (state[s] == 1) {
                    be[2 * nbe] = l;
                    be[2 * nbe + 1] = (uint32_t)s;
                    nbe++;
                } else if (state[s] == 0) {
                    state[s] = 1;
                    stk[sp++] = (uint32_t)s;
                }
            } else {
                state[l] = 2;
                --sp;
            }
        }
        uint8_t *body = (uint8_t *)tmp.alloc(nl, 16);
        if (!body) return false;
        for (uint32_t e = 0; e < nbe; ++e) {
            uint32_t src = be[2 * e], hdr = be[2 * e + 1];
            bool dup = false;
            for (uint32_t f = 0; f < e && !dup; ++f) dup = be[2 * f] == src && be[2 * f + 1] == hdr;
            if (dup) continue;
            for (uint32_t l = 0; l < nl; ++l) body[l] = 0;
            body[hdr] = 1;
            uint32_t sp2 = 0;
            stk[sp2++] = src;
            while (sp2) {
                uint32_t c = stk[--sp2];
                if (body[c]) continue;
                body[c] = 1;
                for (uint32_t q = pcnt[c]; q < pcnt[c + 1]; ++q)
                    if (!body[pred[q]] && sp2 < stk_cap) stk[sp2++] = pred[q];
            }
            uint32_t viol = 0, vl = 0;
            for (uint32_t l = 0; l < nl; ++l)
                if (body[l] && l != hdr && reach[l] && !dominates(hdr, l)) {
                    viol++;
                    vl = l;
                }
            if (viol > 1) {
                unsup = true;  // their order is a Python set's
                return false;
            }
            if (viol == 1) {
                o.put('[');
                o.put(k.name);
                o.put("] non-natural loop: header ");
                put_repr(names[hdr]);
                o.put(" does not dominate reachable body block ");
                put_repr(names[vl]);
                o.put('\n');
            }
        }
        if (o.n == mark1) o.n = mark0;  // no violations: no entry for this kernel
        return true;
    }
    OCB_HD Block &B(uint32_t b) { return m.blocks[b]; }
};

// verify_module(module, check_reachability) as text; false when the TU is
// outside what the verifier reproduces (or scratch ran out).
OCB_HD inline bool verify_module(Module &m, Arena &tmp, Out &o, bool check_reach) {
    Verifier v(m, tmp, o);
    for (uint32_t ki = 0; ki < m.kernels.n; ++ki) {
        uint64_t mark = tmp.used;
        bool ok = v.kernel(m.kernels[ki], check_reach);
        tmp.used = mark;
        if (!ok) return false;
    }
    return true;
}

}  // namespace cc
}  // namespace ocb
