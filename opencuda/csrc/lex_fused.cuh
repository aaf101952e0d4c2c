// Single-pass batch lexer for sm_100a: one kernel reads each source byte from
// HBM once and writes each token record once.
//
// Restates opencuda/frontend/lexer.py:258-295 (lex) for every TU of a batch,
// with the segmentation of lex_kernels.cuh (mode automaton -> sync points ->
// token automaton between sync points), fused per tile of 8 KiB:
//   1. each of the CTA's 256 threads takes a 32-byte window and builds the
//      transition map of the 8-state mode automaton over it;
//   2. a block scan composes the maps; a decoupled look-back over the tiles
//      before this one gives the mode state at the tile start, so every
//      window knows its start state;
//   3. each thread walks its window from that state to its first sync point
//      (a provable token boundary), stopping early; one thread walks past
//      the tile end to the first sync point there, which closes the tile's
//      last segment (and is exactly where the next tile's first segment
//      starts);
//   4. a block suffix-min turns first sync points into segments; each thread
//      runs the token automaton over its segment once, buffering up to FB
//      token records in shared memory and counting the rest;
//   5. a block scan of the counts and a second decoupled look-back give the
//      tile's first output index; warps copy the buffered records out in
//      coalesced order.  A thread whose segment held more than FB tokens
//      lexes it again, writing straight to global memory.
// Tiles are taken in order from an atomic ticket, so a tile only ever waits
// for tiles that already run.  Every wait is bounded: after LB_SPIN_LIMIT
// polls the tile records an error (the host then fails the call) and
// publishes an error word so no later tile waits on it.
//
// Token records: start (u32) and kind << 24 | len (u32); this kernel does
// not produce the per-token line (callers that need it use the multi-pass
// pipeline of lex.cu).
#pragma once
#include "lex_kernels.cuh"

namespace ocb {
namespace lex {

constexpr int FT = 256;                          // threads = windows per tile
constexpr uint64_t FTILE = (uint64_t)FT * WIN;   // source bytes per tile
constexpr int FB = 16;                           // token records buffered per thread
constexpr int FMIN_BLOCKS = 4;                   // resident CTAs per SM requested

// Tile status words of the two look-backs: flag in bits 62-63, payload below.
constexpr uint64_t LB_AGG = 1ull << 62;   // payload: this tile's own aggregate
constexpr uint64_t LB_INC = 2ull << 62;   // payload: inclusive prefix up to this tile
constexpr uint64_t LB_ERR = 3ull << 62;   // a look-back gave up (payload meaningless)
constexpr uint64_t LB_PAY = (1ull << 62) - 1;
constexpr uint32_t LB_SPIN_LIMIT = 1u << 24;

struct FusedArgs {
    const uint8_t *__restrict__ src;
    uint64_t N;
    const uint64_t *__restrict__ tu_off;
    uint32_t n_tu;
    uint64_t n_win, n_tiles;
    unsigned long long *ticket;   // zeroed before the launch
    unsigned long long *mstat;    // n_tiles mode words, zeroed
    unsigned long long *cstat;    // n_tiles count words, zeroed
    unsigned int *err;            // zeroed; set when a look-back gives up
    LexOut o;                     // o.line must be null
    uint64_t *n_tok;
};

// ---- packed mode maps: 3 bits per start state ------------------------------
__device__ __forceinline__ uint32_t map_pack(uint64_t m) {
    uint32_t r = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) r |= (uint32_t)((m >> (8 * s)) & 7u) << (3 * s);
    return r;
}
__device__ __forceinline__ uint32_t pmap_apply(uint32_t pm, uint32_t s) { return (pm >> (3 * s)) & 7u; }
// a then b
__device__ __forceinline__ uint32_t pmap_compose(uint32_t a, uint32_t b) {
    uint32_t r = 0;
#pragma unroll
    for (int s = 0; s < 8; ++s) r |= pmap_apply(b, pmap_apply(a, s)) << (3 * s);
    return r;
}
constexpr uint32_t PMAP_IDENTITY = 0 | 1 << 3 | 2 << 6 | 3 << 9 | 4 << 12 | 5 << 15 | 6 << 18 | 7 << 21;

__device__ __forceinline__ uint64_t lb_load(const unsigned long long *p) {
    return *(const volatile unsigned long long *)p;
}
__device__ __forceinline__ void lb_store(unsigned long long *p, uint64_t v) {
    *(volatile unsigned long long *)p = v;
}

// Warp-wide look-back window: lane L holds the status word of tile
// base - L (tiles before tile 0 read as an inclusive word with payload 0).
// Re-reads until every lane up to the closest inclusive word has published;
// returns that lane (32 when the window holds none).  Bounded: after
// LB_SPIN_LIMIT polls it records the error and returns -1.
__device__ __forceinline__ int lb_window(unsigned long long *stat, int64_t base, uint32_t lane,
                                         unsigned int *err, uint64_t &v) {
    uint32_t spins = 0;
    for (;;) {
        int64_t j = base - (int64_t)lane;
        v = j >= 0 ? lb_load(stat + j) : LB_INC;
        uint32_t f = (uint32_t)(v >> 62);
        unsigned inc = __ballot_sync(0xFFFFFFFFu, f >= 2);   // inclusive or error
        unsigned zero = __ballot_sync(0xFFFFFFFFu, f == 0);
        int first = inc ? __ffs(inc) - 1 : 32;
        unsigned need = first == 32 ? 0xFFFFFFFFu : ((2u << first) - 1u);
        if (!(zero & need)) return first;
        if (++spins > LB_SPIN_LIMIT) {
            if (lane == 0) atomicExch(err, 1u);
            return -1;
        }
        __nanosleep(64);
    }
}

// Mode state at the start of `tile` (whose own map is `agg`): publishes the
// aggregate, looks back 32 tiles at a time, publishes the inclusive end
// state.  Called by all lanes of one warp.
__device__ uint32_t lookback_mode(const FusedArgs &A, uint64_t tile, uint32_t agg,
                                  uint32_t lane) {
    if (tile == 0) {
        if (lane == 0) lb_store(A.mstat, LB_INC | pmap_apply(agg, S_CODE));
        return S_CODE;
    }
    if (lane == 0) lb_store(A.mstat + tile, LB_AGG | agg);
    __syncwarp();
    uint32_t acc = PMAP_IDENTITY;  // maps of the tiles after the inclusive one
    uint32_t s_in = S_CODE;
    bool bad = false;
    for (int64_t base = (int64_t)tile - 1;; base -= 32) {
        uint64_t v;
        int first = lb_window(A.mstat, base, lane, A.err, v);
        if (first < 0) { bad = true; break; }
        // apply the window's maps, oldest first: lanes first-1 .. 0 (or 31 .. 0)
        uint32_t win = PMAP_IDENTITY;
        for (int L = (first == 32 ? 31 : first - 1); L >= 0; --L)
            win = pmap_compose(win, (uint32_t)__shfl_sync(0xFFFFFFFFu, (uint32_t)(v & 0xFFFFFFu), L));
        acc = pmap_compose(win, acc);
        if (first < 32) {
            uint64_t vf = __shfl_sync(0xFFFFFFFFu, v, first);
            if ((vf >> 62) == 3) bad = true;
            else s_in = pmap_apply(acc, (uint32_t)(vf & 7u));
            break;
        }
    }
    if (lane == 0) lb_store(A.mstat + tile, bad ? LB_ERR : (LB_INC | pmap_apply(agg, s_in)));
    return s_in;
}

// First output index of `tile` (whose own count is `cnt`); all lanes of one
// warp, 32 predecessors per probe.
__device__ uint64_t lookback_count(const FusedArgs &A, uint64_t tile, uint64_t cnt, uint32_t lane) {
    if (tile == 0) {
        if (lane == 0) lb_store(A.cstat, LB_INC | cnt);
        return 0;
    }
    if (lane == 0) lb_store(A.cstat + tile, LB_AGG | cnt);
    __syncwarp();
    uint64_t acc = 0;
    bool bad = false;
    for (int64_t base = (int64_t)tile - 1;; base -= 32) {
        uint64_t v;
        int first = lb_window(A.cstat, base, lane, A.err, v);
        if (first < 0) { bad = true; break; }
        uint64_t x = (first == 32 || (int)lane <= first) ? (v & LB_PAY) : 0;
#pragma unroll
        for (int d = 16; d >= 1; d >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, d);
        acc += x;
        if (first < 32) {
            if ((__shfl_sync(0xFFFFFFFFu, v, first) >> 62) == 3) bad = true;
            break;
        }
    }
    if (lane == 0) lb_store(A.cstat + tile, bad ? LB_ERR : (LB_INC | (acc + cnt)));
    return acc;
}

// TU boundary masks of the span [base, base+40) (as window_masks), searching
// only TUs klo..khi (the TUs that touch the tile).
__device__ __forceinline__ void window_masks_in(const uint64_t *tu_off, uint32_t n_tu, uint64_t N,
                                                uint64_t base, uint32_t klo, uint32_t khi,
                                                uint64_t &tus, uint64_t &bnd) {
    tus = 0;
    bnd = 0;
    uint32_t lo = klo, hi = khi;  // first k in [klo, khi] with tu_off[k] >= base
    while (lo < hi) {
        uint32_t mid = (lo + hi) >> 1;
        if (__ldg(tu_off + mid) < base) lo = mid + 1; else hi = mid;
    }
    for (uint32_t k = lo; k <= n_tu; ++k) {
        uint64_t x = __ldg(tu_off + k);
        if (x >= base + 40) break;
        uint64_t bit = 1ull << (x - base);
        bnd |= bit;
        if (k < n_tu && x < N) tus |= bit;
    }
}

// Mode-automaton class of byte q (runtime index; same as class_at): `e` is the
// end of q's TU.
__device__ __forceinline__ uint32_t class_rt(const uint8_t *src, uint64_t q, uint64_t e) {
    uint32_t c = __ldg(src + q);
    if (c != '\n' && c != '/' && c != '*' && c != '\'' && c != '"') return C_OTHER;
    uint64_t left = e - q - 1;
    int nv = left >= 3 ? 3 : (int)left;
    uint32_t n1 = nv >= 1 ? __ldg(src + q + 1) : 0u;
    uint32_t n2 = nv >= 2 ? __ldg(src + q + 2) : 0u;
    uint32_t n3 = nv >= 3 ? __ldg(src + q + 3) : 0u;
    int odd = (c == '"' && q > 0 && __ldg(src + q - 1) == '\\') ? backslash_run_odd(src, q) : 0;
    return classify(c, n1, n2, n3, nv, odd);
}

// First sync point at or after `q`, entering q in mode state `st` (the rules
// of k_lex_sync: a TU start, or the position after a whitespace byte read in
// CODE, or after the newline that ends a // comment); N when there is none.
// `k` is the TU holding q.  Bounded by `lim` bytes (returns NO_SYNC beyond).
__device__ uint64_t first_sync_from(const uint8_t *src, uint64_t N, const uint64_t *tu_off,
                                    uint32_t n_tu, uint64_t q, uint32_t st, uint32_t k,
                                    uint64_t lim) {
    // k is the last TU that starts at or before q: a TU starting exactly at
    // q holds bytes (q < N), so q itself is a sync point
    if (__ldg(tu_off + k) == q) return q;
    uint64_t e = __ldg(tu_off + k + 1);
    uint64_t stop = lim < N ? lim : N;
    for (; q < stop; ++q) {
        while (q == e && k < n_tu) {  // q starts TU k+1 (or a run of empty TUs)
            ++k;
            e = k < n_tu ? __ldg(tu_off + k + 1) : N;
            if (q < N && q < e) return q;
            st = S_CODE;
        }
        uint32_t c = __ldg(src + q);
        if ((st == S_CODE && (c == ' ' || c == '\t' || c == '\r' || c == '\n')) ||
            (st == S_LC && c == '\n'))
            return q + 1;
        st = next_state(c_tsel[class_rt(src, q, e)], st);
    }
    return q >= N ? N : NO_SYNC;
}

// The token automaton over [a, b) (a sync point), as dfa_segment<true>,
// buffering the first FB records in shared memory (slot j*FT + tid).
// Returns the number of records; *k_first receives the TU of its first EOF.
__device__ uint32_t dfa_segment_buf(ByteWin &bw, const uint64_t *__restrict__ tu_off,
                                    uint32_t n_tu, uint64_t a, uint64_t b, const KwPacked *kw,
                                    const DfaSmem &T, const LexOut &o, uint32_t *s_start,
                                    uint32_t *s_kl, uint32_t tid, uint32_t &k_first) {
    uint32_t n = 0;
    uint32_t k = upper_bound_u64(tu_off, n_tu, a) - 1;
    k_first = a == 0 ? 0 : k;
    auto emit = [&](uint32_t pos, uint32_t kind, uint32_t len) {
        if (n < (uint32_t)FB) {
            s_start[n * FT + tid] = pos;
            s_kl[n * FT + tid] = (kind << 24) | len;
        }
        n++;
    };
    if (a == 0)
        for (uint32_t j = 0; j < k; ++j) emit(0, K_EOF, 0);
    uint32_t e = (uint32_t)__ldg(tu_off + k + 1);
    const uint32_t b32 = (uint32_t)b;
    uint32_t tok = (uint32_t)a, q = (uint32_t)a, last = (uint32_t)a;
    uint32_t st = Q_START, lk = 0;
    uint64_t w0 = 0, w1 = 0;
    for (;;) {
        if (st == Q_START) {
            while (tok == e && e <= b32) {
                emit(e, K_EOF, 0);
                ++k;
                if (k >= n_tu) break;
                e = (uint32_t)__ldg(tu_off + k + 1);
            }
            if (k >= n_tu || tok >= b32) break;
        }
        bool in_tu = q < e;
        uint32_t c = in_tu ? bw.at(q) : 0u;
        uint32_t cls = in_tu ? T.cls[c] : (uint32_t)B_EOT;
        uint32_t ns = T.next[st * NB + cls];
        uint32_t ac = T.acc[ns];
        bool adv = ns != Q_DEAD;
        bool has = lk != 0;
        if (!adv && has && lk != ACC_SKIP) {
            uint32_t kind = lk;
            uint32_t L = last - tok;
            if (kind == K_IDENT) kind = keyword_kind_packed(w0, w1, L, kw);
            if (kind & HEXFLOAT) {
                uint32_t v = hexfloat_verdict(Src{bw.src}, tok, L);
                if (v) atomicMin(o.errkey + k, (unsigned long long)(((uint64_t)tok << 8) | v));
            }
            if (L > 0xFFFFFFu) o.unsup[k] = 1;
            emit(tok, kind, L > 0xFFFFFFu ? 0xFFFFFFu : L);
        }
        uint32_t ntok = has ? last : tok + 1;
        uint32_t q1 = q + 1;
        bool acc_now = adv && ac != 0;
        uint32_t j = q - tok;
        uint64_t cb = (uint64_t)c;
        w0 |= (adv && j < 8) ? cb << (8 * j) : 0ull;
        w1 |= (adv && j >= 8 && j < 16) ? cb << (8 * (j - 8)) : 0ull;
        w0 = adv ? w0 : 0ull;
        w1 = adv ? w1 : 0ull;
        last = acc_now ? q1 : (adv ? last : ntok);
        lk = acc_now ? ac : (adv ? lk : 0u);
        st = adv ? ns : (uint32_t)Q_START;
        tok = adv ? tok : ntok;
        q = adv ? q1 : ntok;
    }
    return n;
}

__global__ void __launch_bounds__(FT, FMIN_BLOCKS) k_lex_fused(FusedArgs A) {
    __shared__ DfaSmem T;
    __shared__ KwPacked kwp[128];
    __shared__ uint32_t s_start[FB * FT];
    __shared__ uint32_t s_kl[FB * FT];
    __shared__ uint64_t s_sync[FT + 1];
    __shared__ uint64_t s_wmap[FT / 32];
    __shared__ uint64_t s_wmin[FT / 32];
    __shared__ uint32_t s_wcnt[FT / 32 + 1];
    __shared__ uint32_t s_excl[FT + 1];
    __shared__ uint64_t s_tile, s_tile_off;
    __shared__ uint32_t s_klo, s_khi, s_state_in, s_agg;
    load_kw_packed(kwp, g_kw);
    load_dfa(T);
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (;;) {
        if (tid == 0) s_tile = atomicAdd(A.ticket, 1ull);
        __syncthreads();
        const uint64_t tile = s_tile;
        if (tile >= A.n_tiles) break;
        const uint64_t tbase = tile * FTILE;
        const uint64_t tend = tbase + FTILE < A.N ? tbase + FTILE : A.N;
        if (tid == 0) {
            s_klo = upper_bound_u64(A.tu_off, A.n_tu + 1, tbase) - 1;
            s_khi = upper_bound_u64(A.tu_off, A.n_tu + 1, tbase + FTILE + 40);
            if (s_khi > A.n_tu) s_khi = A.n_tu;
        }
        __syncthreads();
        // 1. window map
        const uint64_t w = tile * FT + tid;
        const uint64_t base = w * WIN;
        uint64_t tus = 0, bnd = 0;
        uint32_t mlo = 0x03020100u, mhi = 0x07060504u;
        if (w < A.n_win) {
            uint32_t wd[NWORD];
            load_window(A.src, A.N, base, wd);
            window_masks_in(A.tu_off, A.n_tu, A.N, base, s_klo, s_khi, tus, bnd);
            MapStep<WIN - 1>::run(wd, bnd, tus, A.src, base, A.N, mlo, mhi);
        }
        uint64_t m = ((uint64_t)mhi << 32) | mlo;
        // 2. block scan of the maps (inclusive), then the tile's start state
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            uint64_t y = __shfl_up_sync(0xFFFFFFFFu, m, d);
            if (lane >= (uint32_t)d) m = map_compose(y, m);
        }
        if (lane == 31) s_wmap[warp] = m;
        __syncthreads();
        uint64_t wpre = MAP_IDENTITY;
        for (uint32_t q = 0; q < warp; ++q) wpre = map_compose(wpre, s_wmap[q]);
        m = map_compose(wpre, m);                      // inclusive map of window tid
        uint64_t mx = __shfl_up_sync(0xFFFFFFFFu, m, 1);
        if (lane == 0) mx = wpre;                      // exclusive map
        if (tid == FT - 1) s_agg = map_pack(m);
        __syncthreads();
        if (warp == 0) {
            uint32_t si = lookback_mode(A, tile, s_agg, lane);
            if (lane == 0) s_state_in = si;
        }
        __syncthreads();
        const uint32_t s_in = s_state_in;
        uint32_t st0 = (uint32_t)((mx >> (8 * s_in)) & 0xFFu);   // mode at my window start
        // 3. first sync point of the window; the last thread also finds the
        // first one at or after the tile end
        uint64_t fs = NO_SYNC;
        if (w < A.n_win) {
            uint32_t k = upper_bound_u64(A.tu_off, A.n_tu, base) - 1;
            fs = first_sync_from(A.src, A.N, A.tu_off, A.n_tu, base, st0, k, base + WIN);
        }
        s_sync[tid] = fs;
        if (tid == FT - 1) {
            uint64_t sb = A.N;
            if (tend < A.N) {
                uint32_t st_end = (uint32_t)((m >> (8 * s_in)) & 0xFFu);
                uint32_t k = upper_bound_u64(A.tu_off, A.n_tu, tend) - 1;
                sb = first_sync_from(A.src, A.N, A.tu_off, A.n_tu, tend, st_end, k, ~0ull);
            }
            s_sync[FT] = sb;
        }
        __syncthreads();
        // 4. segments: [s_sync[tid], min(s_sync[tid+1..FT])), a suffix min
        // within each warp (shuffles), then over the later warps' minima
        uint64_t nxt;
        {
            uint64_t v = s_sync[tid + 1];
#pragma unroll
            for (int d = 1; d < 32; d <<= 1) {
                uint64_t y = __shfl_down_sync(0xFFFFFFFFu, v, d);
                if (lane + d < 32) v = y < v ? y : v;
            }
            if (lane == 0) s_wmin[warp] = v;   // min over s_sync[32w+1 .. 32w+32]
            __syncthreads();
            uint64_t later = s_sync[FT];
            for (uint32_t q = warp + 1; q < FT / 32; ++q) later = s_wmin[q] < later ? s_wmin[q] : later;
            nxt = v < later ? v : later;
        }
        uint64_t a = fs, b = nxt;
        if (a > A.N) a = A.N;
        if (b > A.N) b = A.N;
        uint32_t n = 0, k_first = 0;
        ByteWin bw{A.src, A.N, ~0ull, make_uint4(0, 0, 0, 0)};
        if (fs != NO_SYNC && a < b)
            n = dfa_segment_buf(bw, A.tu_off, A.n_tu, a, b, kwp, T, A.o, s_start, s_kl, tid,
                                k_first);
        // 5. block exclusive scan of the counts
        uint32_t x = n;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, d);
            if (lane >= (uint32_t)d) x += y;
        }
        if (lane == 31) s_wcnt[warp] = x;
        __syncthreads();
        if (tid == 0) {
            uint32_t run = 0;
            for (uint32_t q = 0; q < FT / 32; ++q) {
                uint32_t t = s_wcnt[q];
                s_wcnt[q] = run;
                run += t;
            }
            s_wcnt[FT / 32] = run;
        }
        __syncthreads();
        const uint32_t excl = s_wcnt[warp] + x - n;
        s_excl[tid] = excl;
        if (tid == FT - 1) s_excl[FT] = s_wcnt[FT / 32];
        __syncthreads();
        if (warp == 0) {
            uint64_t off = lookback_count(A, tile, s_wcnt[FT / 32], lane);
            if (lane == 0) s_tile_off = off;
        }
        __syncthreads();
        const uint64_t out0 = s_tile_off;
        // coalesced copy of the buffered records, warp by warp
        {
            const uint32_t w_lo = s_excl[32 * warp], w_hi = s_excl[32 * warp + 32];
            for (uint32_t i = w_lo + lane; i < w_hi; i += 32) {
                uint32_t lo = 32 * warp, hi = 32 * warp + 32;   // owner: last t with excl[t] <= i
                while (hi - lo > 1) {
                    uint32_t mid = (lo + hi) >> 1;
                    if (s_excl[mid] <= i) lo = mid; else hi = mid;
                }
                uint32_t t = lo, jj = i - s_excl[t];
                uint32_t nt = s_excl[t + 1] - s_excl[t];
                if (nt > (uint32_t)FB) continue;   // that thread writes its own records
                uint64_t gi = out0 + i;
                if (gi < A.o.cap) {
                    A.o.start[gi] = s_start[jj * FT + t];
                    A.o.kindlen[gi] = s_kl[jj * FT + t];
                }
            }
        }
        // per-TU token offsets at the EOF records, and the overflowing threads
        if (n > (uint32_t)FB) {
            uint64_t nn = dfa_segment<true>(bw, A.tu_off, A.n_tu, a, b, 1u, kwp, T, out0 + excl,
                                            A.o);
            (void)nn;
        } else {
            uint32_t kk = k_first;
            for (uint32_t j = 0; j < n; ++j)
                if ((s_kl[j * FT + tid] >> 24) == K_EOF) {
                    A.o.tu_tok_off[kk + 1] = out0 + excl + j + 1;
                    ++kk;
                }
        }
        if (tile == A.n_tiles - 1 && tid == 0) {
            *A.n_tok = out0 + s_excl[FT];
            A.o.tu_tok_off[0] = 0;
        }
        __syncthreads();   // shared buffers are reused by the next tile
    }
}

// Per-TU statuses of the fused lexer (as k_lex_finish): every TU reports
// OCB_TU_TIMEOUT when a look-back gave up.
__global__ void k_lex_fused_finish(uint32_t n_tu, const unsigned long long *errkey,
                                   const uint32_t *unsup, const unsigned int *err,
                                   int32_t *status) {
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_tu) {
        int32_t st = 0;
        if (*err) st = OCB_TU_TIMEOUT;
        else if (unsup[i]) st = OCB_TU_UNSUPPORTED;
        else if (errkey[i] != ~0ull) st = (int32_t)(errkey[i] & 0xFFu);
        status[i] = st;
    }
}

}  // namespace lex
}  // namespace ocb
