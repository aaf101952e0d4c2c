// Single-pass batch lexer (sm_100a): one kernel reads every source byte once.
//
// Same algorithm as the multi-pass pipeline of lex_kernels.cuh (8-state mode
// automaton, sync points, exact sequential matcher between them), fused into
// one kernel over 8 KiB tiles with two decoupled look-backs:
//
//   1. the block stages its tile (+64 bytes of halo) in shared memory with
//      16-byte loads, and the tile's TU boundaries;
//   2. every thread builds the transition map of its 32-byte window; a block
//      scan composes them; look-back #1 over earlier tiles' aggregates gives
//      the mode state at the tile start, hence at every window start;
//   3. each thread finds its window's first sync point, a block suffix-min
//      gives its segment [S_t, S_t+1); it lexes the segment with the exact
//      matcher, buffering up to SLOTS tokens in shared memory and counting
//      tokens and the newlines the reference counts (segmented per TU);
//   4. a block scan plus look-back #2 (token count, segmented newlines) give
//      the output index and the line of every token; buffered tokens go out
//      directly, a thread with more than SLOTS tokens re-lexes its segment.
//
// Tiles are taken in order from an atomic ticket so every look-back waits
// only on tiles that are already running or done.  Waits are bounded: after
// ~2 s a block marks its tile poisoned, sets the error word and returns; the
// finishing kernel then reports every TU as OCB_TU_TIMEOUT.
#pragma once
#include "lex_kernels.cuh"

namespace ocb {
namespace lex2 {
using namespace ocb::lex;

constexpr int T = 256;               // threads per block
constexpr int W = 32;                // bytes per thread window
constexpr int TILE = T * W;          // bytes per tile
constexpr int HALO = 64;             // bytes staged past the tile
constexpr int SPAN = TILE + HALO;
constexpr int SLOTS = 16;            // buffered tokens per thread
constexpr int MAXB = 128;            // TU boundaries cached per tile
constexpr long long SPIN_CYCLES = 4000000000ll;

enum : unsigned { F_NONE = 0, F_AGG = 1, F_INC = 2, F_POISON = 3 };

struct TileStatus {
    unsigned flag1, state1;          // look-back #1: flag, inclusive end state
    unsigned long long map1;         // aggregate map of the tile
    unsigned flag2, pad;
    unsigned long long tok_agg, seg_agg, tok_inc, seg_inc;
};

struct Lex2Args {
    const uint8_t *src;
    uint64_t N;
    const uint64_t *tu_off;
    uint32_t n_tu;
    uint32_t n_tiles;
    TileStatus *ts;
    unsigned *ticket;
    unsigned *err;
    LexOut o;
    uint64_t *total;  // written by the last tile
};

// Shared-memory layout (dynamic).
struct Smem {
    uint8_t buf[SPAN];
    uint64_t bnd[MAXB];                  // TU boundaries in [base, base+SPAN)
    uint64_t scan[2 * T];
    uint64_t scan2[2 * T];
    uint32_t slot_start[SLOTS * T], slot_kl[SLOTS * T], slot_ln[SLOTS * T];
    uint32_t tile, kb, k_lo, nb;         // kb: TU containing base; k_lo: first boundary index
    int bnd_ok;
    uint32_t start_state, poisoned;
    unsigned long long tok_prefix, seg_prefix;
    uint64_t next_sync;
};

struct TileSrc {
    const uint8_t *g;
    const uint8_t *sh;
    uint64_t base, span;
    __device__ __forceinline__ uint32_t operator[](uint64_t i) const {
        uint64_t d = i - base;
        return d < span ? (uint32_t)sh[d] : (uint32_t)__ldg(g + i);
    }
};

// Inclusive block scan (Hillis-Steele over shared memory).
template <class Op>
__device__ __forceinline__ uint64_t block_scan(uint64_t x, uint64_t *buf, Op op, bool reverse) {
    int t = reverse ? T - 1 - (int)threadIdx.x : (int)threadIdx.x;
    int cur = 0;
    buf[t] = x;
    __syncthreads();
    for (int d = 1; d < T; d <<= 1) {
        uint64_t y = buf[cur * T + t];
        if (t >= d) y = reverse ? op(y, buf[cur * T + t - d]) : op(buf[cur * T + t - d], y);
        buf[(1 - cur) * T + t] = y;
        cur ^= 1;
        __syncthreads();
    }
    uint64_t r = buf[cur * T + t];
    __syncthreads();
    return r;
}

// Masks of TU boundaries in [pos, pos+40) (bits as in window_masks), from the
// tile's cached list when it covers the range.
__device__ __forceinline__ void masks_at(const Smem &S, const Lex2Args &A, uint64_t base,
                                         uint64_t pos, uint64_t &tus, uint64_t &bnd) {
    if (!S.bnd_ok || pos + 40 > base + SPAN || pos < base) {
        window_masks(A.tu_off, A.n_tu, A.N, pos, tus, bnd);
        return;
    }
    tus = 0;
    bnd = 0;
    for (uint32_t j = 0; j < S.nb; ++j) {
        uint64_t x = S.bnd[j];
        if (x < pos) continue;
        if (x >= pos + 40) break;
        uint64_t bit = 1ull << (x - pos);
        bnd |= bit;
        if (S.k_lo + j < A.n_tu && x < A.N) tus |= bit;
    }
}

// Last TU whose start is <= pos (pos inside the tile's span).
__device__ __forceinline__ uint32_t tu_of(const Smem &S, const Lex2Args &A, uint64_t pos) {
    if (!S.bnd_ok) return upper_bound_u64(A.tu_off, A.n_tu, pos) - 1;
    uint32_t k = S.kb;
    for (uint32_t j = 0; j < S.nb; ++j) {
        if (S.bnd[j] > pos) break;
        if (S.k_lo + j < A.n_tu) k = S.k_lo + j;
    }
    return k;
}

// Class of the byte at q, any position (slow path: global memory, search).
__device__ __noinline__ uint32_t class_global(const Lex2Args &A, uint64_t q) {
    uint32_t c = __ldg(A.src + q);
    if (c != '\n' && c != '/' && c != '*' && c != '\'' && c != '"') return C_OTHER;
    uint64_t tus, bnd;
    window_masks(A.tu_off, A.n_tu, A.N, q, tus, bnd);
    int nv = ((bnd >> 1) & 1) ? 0 : ((bnd >> 2) & 1) ? 1 : ((bnd >> 3) & 1) ? 2 : 3;
    uint32_t n1 = nv >= 1 ? __ldg(A.src + q + 1) : 0, n2 = nv >= 2 ? __ldg(A.src + q + 2) : 0,
             n3 = nv >= 3 ? __ldg(A.src + q + 3) : 0;
    int odd = c == '"' ? backslash_run_odd(A.src, q) : 0;
    return classify(c, n1, n2, n3, nv, odd);
}

// Sync predicate after byte c read in state st.
__device__ __forceinline__ bool sync_after(uint32_t st, uint32_t c) {
    return (st == S_CODE && (c == ' ' || c == '\t' || c == '\r' || c == '\n')) ||
           (st == S_LC && c == '\n');
}

// First sync point at or after `from` when the state at `from` is st; walks
// global memory (used only past the tile).  Returns N if none.
__device__ __noinline__ uint64_t find_sync_global(const Lex2Args &A, uint64_t from, uint32_t st,
                                                  const uint32_t *tsel) {
    uint64_t q = from;
    if (q >= A.N) return A.N;
    uint32_t k = upper_bound_u64(A.tu_off, A.n_tu, q) - 1;
    uint64_t tu_start = __ldg(A.tu_off + k);
    if (tu_start == q) return q;
    uint64_t next_b = __ldg(A.tu_off + k + 1);
    while (q < A.N) {
        if (q == next_b) return q;  // a TU start (boundaries are sync points)
        uint32_t c = __ldg(A.src + q);
        uint32_t cls = class_global(A, q);
        if (sync_after(st, c)) return q + 1;
        st = next_state(tsel[cls], st);
        ++q;
    }
    return A.N;
}

__device__ __forceinline__ bool wait_flag(volatile unsigned *f, unsigned &v, long long t0) {
    for (unsigned it = 0;; ++it) {
        v = *f;
        if (v != F_NONE) return true;
        if ((it & 31) == 31 && clock64() - t0 > SPIN_CYCLES) return false;
        __nanosleep(100);
    }
}

// Lex [a, b) buffering tokens in the thread's shared slots.  Lines are kept
// relative: a token's slot line is (reset ? 0x80000000 | line : newlines since
// a).  Returns the token count; `seg` receives (flag, newlines since the last
// TU start in the segment, or since a).
__device__ uint32_t lex_seg_buffer(const Lex2Args &A, Smem &S, TileSrc s, uint64_t a, uint64_t b,
                                   uint32_t k, bool a_is_start, uint64_t &seg) {
    const KwEntry *kw = g_kw;
    const uint32_t t = threadIdx.x;
    uint32_t n = 0;
    bool reset = a_is_start;
    uint32_t ln = a_is_start ? 1u : 0u;
    auto put = [&](uint32_t start, uint32_t kl, uint32_t line_code) {
        if (n < SLOTS) {
            S.slot_start[n * T + t] = start;
            S.slot_kl[n * T + t] = kl;
            S.slot_ln[n * T + t] = line_code;
        }
        n++;
    };
    if (a == 0) {
        for (uint32_t j = 0; j < k; ++j) put(j, K_EOF << 24, 0x80000001u);  // empty TUs at 0
    }
    uint64_t p = a, e = __ldg(A.tu_off + k + 1);
    for (;;) {
        while (p == e && e <= b) {
            put(k, K_EOF << 24, reset ? (0x80000000u | ln) : ln);
            ++k;
            reset = true;
            ln = 1;
            if (k >= A.n_tu) break;
            e = __ldg(A.tu_off + k + 1);
        }
        if (k >= A.n_tu || p >= b) break;
        Match m = lex_one(s, p, e, kw);
        if (m.kind != K_NONE) {
            uint32_t kl = (m.kind << 24) | (uint32_t)(m.len > 0xFFFFFFu ? 0xFFFFFFu : m.len);
            put((uint32_t)p, kl, reset ? (0x80000000u | ln) : ln);
            if (m.kind & HEXFLOAT) {
                uint32_t v = hexfloat_verdict(s, p, m.len);
                if (v) atomicMin(A.o.errkey + k, (unsigned long long)((p << 8) | v));
            }
            if (m.len > 0xFFFFFFu) A.o.unsup[k] = 1;
        }
        ln += m.nl;
        p += m.len;
    }
    seg = reset ? (SEG_FLAG | (uint64_t)(ln - 1)) : (uint64_t)ln;
    return n;
}

struct AddOp {
    __device__ __forceinline__ uint64_t operator()(uint64_t x, uint64_t y) const { return x + y; }
};

// Exclusive value of an inclusive block scan (the previous thread's value).
__device__ __forceinline__ uint64_t exclusive_of(uint64_t inc, uint64_t *buf, uint64_t identity) {
    buf[threadIdx.x] = inc;
    __syncthreads();
    uint64_t r = threadIdx.x ? buf[threadIdx.x - 1] : identity;
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(T) k_lex2(Lex2Args A) {
    extern __shared__ __align__(16) uint8_t smem_raw[];
    Smem &S = *reinterpret_cast<Smem *>(smem_raw);
    __shared__ uint32_t tsel[C_NCLS];
    const uint32_t t = threadIdx.x;
    if (t < C_NCLS) tsel[t] = c_tsel[t];
    if (t == 0) {
        S.tile = atomicAdd(A.ticket, 1u);
        S.poisoned = 0;
    }
    __syncthreads();
    const uint32_t tile = S.tile;
    if (tile >= A.n_tiles) return;
    const uint64_t base = (uint64_t)tile * TILE;
    const uint64_t span = A.N - base < (uint64_t)SPAN ? A.N - base : (uint64_t)SPAN;

    // ---- 1. stage the tile and its TU boundaries ------------------------
    if (span == (uint64_t)SPAN) {
        const uint4 *g = reinterpret_cast<const uint4 *>(A.src + base);
        uint4 *d = reinterpret_cast<uint4 *>(S.buf);
        for (int i = t; i < SPAN / 16; i += T) d[i] = __ldg(g + i);
    } else {
        for (int i = t; i < SPAN; i += T)
            S.buf[i] = (uint64_t)i < span ? __ldg(A.src + base + i) : (uint8_t)0;
    }
    if (t == 0) {
        uint32_t k_lo = lower_bound_u64(A.tu_off, A.n_tu + 1, base);
        uint32_t k_hi = lower_bound_u64(A.tu_off, A.n_tu + 1, base + SPAN);
        S.k_lo = k_lo;
        S.nb = k_hi - k_lo;
        S.bnd_ok = (k_hi - k_lo) <= (uint32_t)MAXB;
        S.kb = upper_bound_u64(A.tu_off, A.n_tu, base) - 1;
    }
    __syncthreads();
    if (S.bnd_ok)
        for (uint32_t j = t; j < S.nb; j += T) S.bnd[j] = __ldg(A.tu_off + S.k_lo + j);
    __syncthreads();

    // ---- 2. window maps, block scan, look-back #1 -------------------------
    const uint64_t w0 = base + (uint64_t)t * W;
    uint64_t tus = 0, bnd = 0;
    masks_at(S, A, base, w0, tus, bnd);
    const uint8_t *wb = S.buf + (size_t)t * W;
    auto cls_local = [&](int i) -> uint32_t {  // class of window byte i
        uint32_t c = wb[i];
        if (c != '\n' && c != '/' && c != '*' && c != '\'' && c != '"') return C_OTHER;
        int nv = ((bnd >> (i + 1)) & 1) ? 0 : ((bnd >> (i + 2)) & 1) ? 1
               : ((bnd >> (i + 3)) & 1) ? 2 : 3;
        int odd = 0;
        if (c == '"') {
            if (i == 0 && t == 0) odd = backslash_run_odd(A.src, w0);
            else if (wb[i - 1] == '\\') odd = backslash_run_odd(A.src, w0 + i);
        }
        return classify(c, wb[i + 1], wb[i + 2], wb[i + 3], nv, odd);
    };
    uint32_t mlo = 0x03020100u, mhi = 0x07060504u;
    if (w0 < A.N) {
        for (int i = W - 1; i >= 0; --i) {
            if (w0 + i >= A.N) continue;
            uint32_t sel = tsel[cls_local(i)];
            uint32_t nlo = __byte_perm(mlo, mhi, sel & 0xFFFFu);
            uint32_t nhi = __byte_perm(mlo, mhi, sel >> 16);
            mlo = nlo;
            mhi = nhi;
            if ((tus >> i) & 1) mlo = mhi = (mlo & 0xFFu) * 0x01010101u;
        }
    }
    const uint64_t inc_map = block_scan(((uint64_t)mhi << 32) | mlo, S.scan, ComposeOp(), false);
    const uint64_t excl_map = exclusive_of(inc_map, S.scan2, MAP_IDENTITY);
    if (t == T - 1) S.scan2[0] = inc_map;
    __syncthreads();
    if (t == 0) {
        const uint64_t agg = S.scan2[0];
        TileStatus *me = A.ts + tile;
        uint32_t start = S_CODE;
        bool ok = true;
        if (tile > 0) {
            me->map1 = agg;
            __threadfence();
            *(volatile unsigned *)&me->flag1 = F_AGG;
            uint64_t acc = MAP_IDENTITY;
            long long t0 = clock64();
            for (int64_t p = (int64_t)tile - 1; p >= 0; --p) {
                unsigned f;
                if (!wait_flag(&A.ts[p].flag1, f, t0) || f == F_POISON) { ok = false; break; }
                __threadfence();
                if (f == F_INC) {
                    uint32_t st0 = *(volatile unsigned *)&A.ts[p].state1;
                    start = (uint32_t)((acc >> (8 * st0)) & 0xFFu);
                    break;
                }
                acc = map_compose(*(volatile unsigned long long *)&A.ts[p].map1, acc);
            }
        }
        if (!ok) {
            S.poisoned = 1;
            atomicOr(A.err, 1u);
            *(volatile unsigned *)&me->flag1 = F_POISON;
            *(volatile unsigned *)&me->flag2 = F_POISON;
        } else {
            me->state1 = (uint32_t)((agg >> (8 * start)) & 0xFFu);
            __threadfence();
            *(volatile unsigned *)&me->flag1 = F_INC;
        }
        S.start_state = start;
    }
    __syncthreads();
    if (S.poisoned) return;
    const uint32_t tile_start = S.start_state;
    uint32_t st = (uint32_t)((excl_map >> (8 * tile_start)) & 0xFFu);

    // ---- 3. first sync point of the window, segments --------------------
    uint64_t fsync = NO_SYNC;
    bool fsync_tu = false;
    for (int i = 0; i < W && w0 + i < A.N; ++i) {
        if ((tus >> i) & 1) {
            fsync = w0 + i;
            fsync_tu = true;
            break;
        }
        uint32_t c = wb[i];
        if (sync_after(st, c)) {
            fsync = w0 + i + 1;
            fsync_tu = (tus >> (i + 1)) & 1;
            break;
        }
        st = next_state(tsel[cls_local(i)], st);
    }
    if (t == T - 1) {
        // the first sync point at or after the next tile, from the tile's end state
        uint64_t nxt = base + TILE, ns = A.N;
        if (nxt < A.N) {
            uint32_t end_state = (uint32_t)((inc_map >> (8 * tile_start)) & 0xFFu);
            ns = find_sync_global(A, nxt, end_state, tsel);
        }
        S.next_sync = ns;
    }
    __syncthreads();
    const uint64_t next_sync = S.next_sync;
    const uint64_t sfx = block_scan(fsync, S.scan, MinOp(), true);  // min over windows >= t
    S.scan2[t] = sfx;
    __syncthreads();
    uint64_t a = sfx < next_sync ? sfx : next_sync;
    uint64_t b = t == T - 1 ? next_sync : S.scan2[t + 1];
    __syncthreads();
    if (b > next_sync) b = next_sync;
    if (a > A.N) a = A.N;
    if (b > A.N) b = A.N;

    // ---- 4. lex the segment (count + buffer) -----------------------------
    TileSrc src{A.src, S.buf, base, span};
    uint32_t ntok = 0;
    uint64_t seg = 0;
    const bool a_is_start = fsync_tu;  // a < b implies a is this window's sync
    if (a < b) ntok = lex_seg_buffer(A, S, src, a, b, tu_of(S, A, a), a_is_start, seg);

    // ---- 5. block scans + look-back #2 ------------------------------------
    const uint64_t tok_inc = block_scan((uint64_t)ntok, S.scan, AddOp(), false);
    const uint64_t seg_inc = block_scan(seg, S.scan, SegSumOp(), false);
    const uint64_t seg_excl = exclusive_of(seg_inc, S.scan2, 0);
    if (t == T - 1) {
        S.scan2[0] = tok_inc;
        S.scan2[1] = seg_inc;
    }
    __syncthreads();
    if (t == 0) {
        const uint64_t tok_agg = S.scan2[0], seg_agg = S.scan2[1];
        TileStatus *me = A.ts + tile;
        uint64_t tok_pre = 0, seg_pre = 0;
        bool ok = true;
        if (tile > 0) {
            me->tok_agg = tok_agg;
            me->seg_agg = seg_agg;
            __threadfence();
            *(volatile unsigned *)&me->flag2 = F_AGG;
            long long t0 = clock64();
            for (int64_t p = (int64_t)tile - 1; p >= 0; --p) {
                unsigned f;
                if (!wait_flag(&A.ts[p].flag2, f, t0) || f == F_POISON) { ok = false; break; }
                __threadfence();
                if (f == F_INC) {
                    tok_pre += *(volatile unsigned long long *)&A.ts[p].tok_inc;
                    seg_pre = SegSumOp()(*(volatile unsigned long long *)&A.ts[p].seg_inc, seg_pre);
                    break;
                }
                tok_pre += *(volatile unsigned long long *)&A.ts[p].tok_agg;
                seg_pre = SegSumOp()(*(volatile unsigned long long *)&A.ts[p].seg_agg, seg_pre);
            }
        }
        if (!ok) {
            S.poisoned = 1;
            atomicOr(A.err, 1u);
            *(volatile unsigned *)&me->flag2 = F_POISON;
        } else {
            me->tok_inc = tok_pre + tok_agg;
            me->seg_inc = SegSumOp()(seg_pre, seg_agg);
            __threadfence();
            *(volatile unsigned *)&me->flag2 = F_INC;
            if (tile == A.n_tiles - 1) *A.total = tok_pre + tok_agg;
        }
        S.tok_prefix = tok_pre;
        S.seg_prefix = seg_pre;
    }
    __syncthreads();
    if (S.poisoned || ntok == 0) return;

    // ---- 6. write the tokens ----------------------------------------------
    const uint64_t out0 = S.tok_prefix + tok_inc - ntok;
    const uint64_t pre = SegSumOp()(S.seg_prefix, seg_excl);
    const uint32_t line_base = a_is_start ? 1u : 1u + (uint32_t)(pre & ~SEG_FLAG);
    if (ntok > (uint32_t)SLOTS) {
        // too many tokens to buffer: lex the segment again, writing directly
        lex_segment<true>(Src{A.src}, A.tu_off, A.n_tu, a, b, line_base, g_kw, out0, A.o);
        return;
    }
    for (uint32_t j = 0; j < ntok; ++j) {
        uint64_t i = out0 + j;
        uint32_t kl = S.slot_kl[j * T + t], start = S.slot_start[j * T + t];
        uint32_t lc = S.slot_ln[j * T + t];
        uint32_t line = (lc & 0x80000000u) ? (lc & 0x7FFFFFFFu) : line_base + lc;
        if ((kl >> 24) == K_EOF) {
            uint32_t k = start;
            start = (uint32_t)__ldg(A.tu_off + k + 1);
            A.o.tu_tok_off[k + 1] = i + 1;
        }
        if (i < A.o.cap) {
            A.o.start[i] = start;
            A.o.kindlen[i] = kl;
            if (A.o.line) A.o.line[i] = line;
        }
    }
}

__global__ void k_lex2_finish(uint32_t n_tu, const unsigned long long *errkey,
                              const uint32_t *unsup, const unsigned *err, int32_t *status,
                              uint64_t *tu_tok_off, const uint64_t *total, uint64_t *n_tok) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_tu) {
        int32_t st = 0;
        if (*err) st = OCB_TU_TIMEOUT;
        else if (unsup[i]) st = OCB_TU_UNSUPPORTED;
        else if (errkey[i] != ~0ull) st = (int32_t)(errkey[i] & 0xFFu);
        status[i] = st;
    }
    if (i == 0) {
        tu_tok_off[0] = 0;
        *n_tok = *err ? 0 : *total;
    }
}

}  // namespace lex2
}  // namespace ocb
