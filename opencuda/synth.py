"""Seeded synthetic CUDA-C workloads for the batch compiler.

Five workload shapes are used by the tests and by ``bench.py``:

* ``sgemm``       -- one tiled SGEMM kernel (16x16 ``__shared__`` tiles,
                     K-tile loop, two ``__syncthreads``, bounds checks).
* ``random``      -- seeded random kernels of 50-200 statements (about 4 KB):
                     60% s32 / 40% f32 arithmetic, if/else nesting <= 3,
                     ``for`` loops of trip count 2-16 with straight-line
                     bodies, 5% ``atomicAdd``, 5% ``__shfl_sync``.
* ``lexstress``   -- preprocessor/lexer stress text: 16 KiB TUs, identifiers
                     ``v{k}`` with k ~ Zipf(1.1) over 10k names, 5% ``#define``
                     lines (half object-like, half function-like), hex, float
                     and suffixed literals, 10% ``//`` and ``/* */`` comments.
* ``regpressure`` -- straight-line kernels with ~20k SSA values and 8 if/else
                     diamonds (40% f32, 30% s32, 20% u64 address math, 10%
                     predicates).
* ``lognormal``   -- ``random`` kernels whose sizes follow a lognormal
                     distribution (median 3 KB, sigma 1).

Every TU is generated from ``random.Random(seed + i)`` so any TU can be
regenerated on its own.  All text is ASCII.
"""
from __future__ import annotations

import random
import numpy as np

# 2: lognormal statement counts calibrated so the byte sizes have the stated
#    median (head and tail ~408 bytes, ~34 bytes per statement)
GEN_VERSION = 2

SGEMM_SRC = r"""// Tiled single-precision GEMM: C = alpha * A * B + beta * C
// A is MxK, B is KxN, C is MxN, all row-major; one 16x16 tile of C per block.
// Each K-step stages one tile of A and one of B in shared memory, with
// out-of-range elements filled with zero, then accumulates their product.
#define TILE 16

__global__ void sgemm_tiled(float *C, const float *A, const float *B,
                            int M, int N, int K, float alpha, float beta) {
    __shared__ float As[TILE][TILE];
    __shared__ float Bs[TILE][TILE];

    int tx = threadIdx.x;
    int ty = threadIdx.y;
    int row = blockIdx.y * TILE + ty;
    int col = blockIdx.x * TILE + tx;

    float acc = 0.0f;
    int numTiles = (K + TILE - 1) / TILE;

    for (int t = 0; t < numTiles; t++) {
        int aCol = t * TILE + tx;
        int bRow = t * TILE + ty;

        // Guarded loads: out-of-range elements are filled with zero.
        if (row < M && aCol < K) {
            As[ty][tx] = A[row * K + aCol];
        } else {
            As[ty][tx] = 0.0f;
        }
        if (bRow < K && col < N) {
            Bs[ty][tx] = B[bRow * N + col];
        } else {
            Bs[ty][tx] = 0.0f;
        }

        __syncthreads();

        for (int k = 0; k < TILE; k++) {
            acc += As[ty][k] * Bs[k][tx];
        }

        __syncthreads();
    }

    // Guarded epilogue.
    if (row < M && col < N) {
        C[row * N + col] = alpha * acc + beta * C[row * N + col];
    }
}
"""


# --------------------------------------------------------------------------
# random kernels (statement mix of the 4,096-kernel and lognormal workloads)
# --------------------------------------------------------------------------

class _KernelGen:
    def __init__(self, rng: random.Random, idx: int):
        self.r = rng
        self.idx = idx
        self.ivars = ["i0", "i1", "i2", "i3"]
        self.fvars = ["f0", "f1", "f2", "f3"]
        self.loopvars = 0

    def iatom(self, extra=()):
        r = self.r.random()
        pool = self.ivars + list(extra)
        if r < 0.55:
            return self.r.choice(pool)
        if r < 0.75:
            return str(self.r.randint(0, 255))
        if r < 0.85:
            return "tid"
        return f"ia[(tid + {self.r.randint(0, 63)}) & 1023]"

    def fatom(self):
        r = self.r.random()
        if r < 0.55:
            return self.r.choice(self.fvars)
        if r < 0.8:
            return f"{self.r.randint(0, 99)}.{self.r.randint(0, 99)}f"
        return f"fa[(tid + {self.r.randint(0, 63)}) & 1023]"

    def iexpr(self, depth=0, extra=()):
        if depth >= 2 or self.r.random() < 0.4:
            return self.iatom(extra)
        op = self.r.choice(["+", "-", "*", "&", "|", "^", "+", "*"])
        if self.r.random() < 0.12:
            return f"({self.iexpr(depth + 1, extra)} >> {self.r.randint(1, 7)})"
        return f"({self.iexpr(depth + 1, extra)} {op} {self.iexpr(depth + 1, extra)})"

    def fexpr(self, depth=0):
        if depth >= 2 or self.r.random() < 0.4:
            return self.fatom()
        op = self.r.choice(["+", "-", "*", "+", "*"])
        return f"({self.fexpr(depth + 1)} {op} {self.fexpr(depth + 1)})"

    def cond(self):
        if self.r.random() < 0.6:
            return (f"{self.iatom()} {self.r.choice(['<', '>', '<=', '>=', '==', '!='])} "
                    f"{self.iatom()}")
        return f"{self.r.choice(self.fvars)} {self.r.choice(['<', '>'])} {self.fatom()}"

    def simple_stmt(self, ind, extra=()):
        r = self.r.random()
        if r < 0.05:
            return (f"{ind}atomicAdd(&io[(tid + {self.r.randint(0, 255)}) & 255], "
                    f"{self.r.choice(self.ivars)});")
        if r < 0.10:
            return (f"{ind}{self.r.choice(self.fvars)} = __shfl_sync(0xffffffff, "
                    f"{self.r.choice(self.fvars)}, {self.r.randint(0, 31)});")
        if r < 0.64:
            v = self.r.choice(self.ivars)
            if self.r.random() < 0.3:
                return f"{ind}{v} {self.r.choice(['+=', '^=', '-='])} {self.iexpr(1, extra)};"
            return f"{ind}{v} = {self.iexpr(0, extra)};"
        v = self.r.choice(self.fvars)
        if self.r.random() < 0.3:
            return f"{ind}{v} += {self.fexpr(1)};"
        return f"{ind}{v} = {self.fexpr()};"

    def block(self, n, depth, ind):
        out = []
        while n > 0:
            r = self.r.random()
            if r < 0.12 and depth < 3 and n >= 3:
                k = self.r.randint(1, min(6, n - 1))
                out.append(f"{ind}if ({self.cond()}) {{")
                out.extend(self.block(k, depth + 1, ind + "    "))
                if self.r.random() < 0.5:
                    k2 = self.r.randint(1, 3)
                    out.append(f"{ind}}} else {{")
                    out.extend(self.block(k2, depth + 1, ind + "    "))
                    n -= k2
                out.append(f"{ind}}}")
                n -= k + 1
            elif r < 0.2 and depth < 3 and n >= 2:
                trip = self.r.randint(2, 16)
                j = f"j{self.loopvars}"
                self.loopvars += 1
                k = self.r.randint(1, min(4, n - 1))
                out.append(f"{ind}for (int {j} = 0; {j} < {trip}; {j}++) {{")
                for _ in range(k):
                    out.append(self.simple_stmt(ind + "    ", extra=(j,)))
                out.append(f"{ind}}}")
                n -= k + 1
            else:
                out.append(self.simple_stmt(ind))
                n -= 1
        return out

    def kernel(self, n_stmts: int) -> str:
        name = f"rk{self.idx}"
        head = [
            f"__global__ void {name}(float *fa, int *ia, int *io, float *fout, int *iout) {{",
            "    int tid = blockIdx.x * blockDim.x + threadIdx.x;",
            "    int i0 = ia[tid & 1023];",
            "    int i1 = ia[(tid + 1) & 1023];",
            "    int i2 = tid * 3;",
            "    int i3 = 7;",
            "    float f0 = fa[tid & 1023];",
            "    float f1 = fa[(tid + 1) & 1023];",
            "    float f2 = 0.5f;",
            "    float f3 = 1.0f;",
        ]
        body = self.block(n_stmts, 0, "    ")
        tail = [
            "    fout[tid] = f0 + f1 + f2 + f3;",
            "    iout[tid] = i0 + i1 + i2 + i3;",
            "}",
        ]
        return "\n".join(head + body + tail) + "\n"


def random_kernel(seed: int, idx: int, n_stmts: int | None = None) -> str:
    r = random.Random(seed)
    if n_stmts is None:
        n_stmts = r.randint(50, 200)
    return _KernelGen(r, idx).kernel(n_stmts)


def random_batch(n: int = 4096, seed: int = 1234) -> list[str]:
    return [random_kernel(seed + i, i) for i in range(n)]


def lognormal_kernel(seed: int, idx: int, median: int = 3000, sigma: float = 1.0) -> str:
    """One kernel of the lognormal workload, its size drawn from
    lognormal(median, sigma) bytes."""
    r = random.Random(seed)
    target = median * float(np.exp(sigma * r.gauss(0.0, 1.0)))
    # ~408 bytes of kernel head and tail plus ~34 bytes per statement
    n_stmts = int(min(max(round((target - 408.0) / 34.0), 4), 4000))
    return _KernelGen(r, idx).kernel(n_stmts)


def _lognormal_range(args):
    lo, hi, seed, median, sigma = args
    return [lognormal_kernel(seed + i, i, median, sigma) for i in range(lo, hi)]


def lognormal_batch(n: int = 262144, seed: int = 5678, median: int = 3000,
                    sigma: float = 1.0, procs: int = 1) -> list[str]:
    """Random kernels with byte sizes ~ lognormal(median, sigma).

    ``procs`` > 1 generates in that many ``spawn`` worker processes (the
    262,144-kernel batch takes minutes in one process); the output does not
    depend on it."""
    if procs <= 1 or n < 4096:
        return _lognormal_range((0, n, seed, median, sigma))
    import multiprocessing as mp
    step = (n + 4 * procs - 1) // (4 * procs)
    jobs = [(lo, min(n, lo + step), seed, median, sigma) for lo in range(0, n, step)]
    with mp.get_context("spawn").Pool(procs) as pool:
        parts = pool.map(_lognormal_range, jobs)
    return [k for part in parts for k in part]


# --------------------------------------------------------------------------
# lexer / preprocessor stress text
# --------------------------------------------------------------------------

def _zipf_names(r: random.Random, n: int, s: float = 1.1, vocab: int = 10000):
    # Inverse-CDF sampling of a bounded Zipf(s) over `vocab` names.
    w = 1.0 / np.power(np.arange(1, vocab + 1, dtype=np.float64), s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    u = np.array([r.random() for _ in range(n)])
    return np.searchsorted(cdf, u)


def _literal(r: random.Random) -> str:
    k = r.random()
    if k < 0.30:
        return str(r.randint(0, 100000))
    if k < 0.45:
        return hex(r.randint(0, 1 << 31)).replace("0x", r.choice(["0x", "0X"]))
    if k < 0.65:
        return f"{r.randint(0, 999)}.{r.randint(0, 999)}f"
    if k < 0.72:
        return f"{r.randint(0, 99)}.{r.randint(0, 99)}e{r.choice(['', '+', '-'])}{r.randint(0, 30)}"
    if k < 0.80:
        return f".{r.randint(0, 999)}f"
    if k < 0.88:
        return f"{r.randint(0, 5000)}{r.choice(['u', 'U', 'ULL', 'u', 'L', 'ull'])}"
    if k < 0.93:
        return f"{r.randint(1, 9)}e{r.randint(0, 9)}f"
    if k < 0.97:
        return f"0x{r.randint(1, 15):x}.{r.randint(0, 255):02x}p{r.choice(['', '+', '-'])}{r.randint(0, 9)}f"
    return f"{r.randint(0, 99)}f"


def _stress_pool(seed: int, n_lines: int) -> list[str]:
    r = random.Random(seed)
    names = _zipf_names(r, n_lines * 6)
    ni = iter(names.tolist())
    ops = ["+", "-", "*", "/", "%", "&", "|", "^", "<<", ">>", "<", ">",
           "<=", ">=", "==", "!=", "&&", "||"]
    asg = ["=", "+=", "-=", "*=", "|=", "^=", "<<=", ">>="]
    lines = []
    for _ in range(n_lines):
        k = r.random()
        if k < 0.025:
            lines.append(f"#define M{r.randint(0, 31)} ({_literal(r)} + v{next(ni)})")
        elif k < 0.05:
            lines.append(f"#define F{r.randint(0, 15)}(a, b) ((a) * {_literal(r)} + (b))")
        elif k < 0.10:
            words = " ".join("v%d" % next(ni) for _ in range(r.randint(1, 6)))
            lines.append(f"    // {words} note")
        elif k < 0.15:
            if r.random() < 0.3:
                lines.append(f"    /* block v{next(ni)}\n       spans v{next(ni)} */")
            else:
                lines.append(f"    /* v{next(ni)} * {_literal(r)} */ v{next(ni)}++;")
        elif k < 0.17:
            lines.append(f"    s{r.randint(0, 9)} = \"v{next(ni)} \\\"q\\\" \\n %d\";")
        elif k < 0.18:
            lines.append(f"    c{r.randint(0, 9)} = '{r.choice('abcxyz')}' + '\\n';")
        else:
            terms = [f"v{next(ni)}" if r.random() < 0.6 else _literal(r)
                     for _ in range(r.randint(1, 4))]
            if r.random() < 0.15:
                terms[0] = f"F{r.randint(0, 15)}(v{next(ni)}, {_literal(r)})"
            if r.random() < 0.15:
                terms[-1] = f"M{r.randint(0, 31)}"
            expr = terms[0]
            for t in terms[1:]:
                expr += f" {r.choice(ops)} {t}"
            if r.random() < 0.2:
                expr = f"(v{next(ni)}[{r.randint(0, 63)}] -> x) ? {expr} : v{next(ni)}.y"
            lines.append(f"    v{next(ni)} {r.choice(asg)} {expr};")
    return lines


PART_BYTES = 256 << 20


def lexstress_batch(total_bytes: int = 1 << 30, tu_bytes: int = 16384,
                    seed: int = 99, pool_lines: int = 200_000):
    """Stress text as (buffer bytes, tu_off int64[n+1]).

    TUs are assembled from a seeded pool of lines so that a GiB builds in
    seconds; each TU is cut at a line boundary once it reaches ``tu_bytes``.
    Batches above 256 MiB are built as independent 256 MiB parts (seeds
    seed, seed+1, ...), each larger than the GPU's L2.
    """
    if total_bytes > PART_BYTES:
        bufs, offs, base = [], [np.zeros(1, np.int64)], 0
        left, k = total_bytes, 0
        while left > 0:
            b, o = lexstress_batch(min(left, PART_BYTES), tu_bytes, seed + k, pool_lines)
            bufs.append(b)
            offs.append(o[1:] + base)
            base += len(b)
            left -= PART_BYTES
            k += 1
        return b"".join(bufs), np.concatenate(offs)
    pool = _stress_pool(seed, pool_lines)
    enc = [(l + "\n").encode() for l in pool]
    lens = np.array([len(e) for e in enc], dtype=np.int64)
    rs = np.random.default_rng(seed)
    mean = float(lens.mean())
    n_pick = int(total_bytes / mean * 1.02) + 16
    pick = rs.integers(0, len(enc), size=n_pick)
    plen = lens[pick]
    cum = np.cumsum(plen)
    n_keep = int(np.searchsorted(cum, total_bytes, side="right"))
    pick, plen, cum = pick[:n_keep], plen[:n_keep], cum[:n_keep]
    total = int(cum[-1]) if n_keep else 0
    # Gather the picked lines into one buffer.
    out = b"".join(map(enc.__getitem__, pick.tolist()))
    # TU cuts at the first line end at or past each tu_bytes boundary.
    cuts = [0]
    target = tu_bytes
    while target < total:
        j = int(np.searchsorted(cum, target, side="left"))
        if j >= len(cum):
            break
        c = int(cum[j])
        if c >= total:
            break
        cuts.append(c)
        target = c + tu_bytes
    cuts.append(total)
    return out, np.array(cuts, dtype=np.int64)


# --------------------------------------------------------------------------
# register-pressure kernels
# --------------------------------------------------------------------------

def regpressure_kernel(seed: int, idx: int, n_stmts: int = 6000) -> str:
    r = random.Random(seed)
    lines = [f"__global__ void rp{idx}(float *fa, int *ia, float *fo, int *io, int n) {{",
             "    int tid = blockIdx.x * blockDim.x + threadIdx.x;"]
    fv, iv, av, pv = [], [], [], []
    diamonds = sorted(r.sample(range(n_stmts), 8))
    for s in range(n_stmts):
        if diamonds and s == diamonds[0]:
            diamonds.pop(0)
            a = r.choice(iv) if iv else "tid"
            lines.append(f"    if ({a} > {r.randint(0, 100)}) {{")
            if fv:
                v = r.choice(fv)
                lines.append(f"        {v} = {v} * 0.5f;")
            lines.append("    } else {")
            if fv:
                v = r.choice(fv)
                lines.append(f"        {v} = {v} + 1.0f;")
            lines.append("    }")
            continue
        k = r.random()
        if k < 0.4:
            name = f"x{len(fv)}"
            if len(fv) >= 2:
                e = f"{r.choice(fv)} {r.choice(['+', '*', '-'])} {r.choice(fv)}"
            else:
                e = f"fa[(tid + {s}) & 4095]"
            lines.append(f"    float {name} = {e};")
            fv.append(name)
        elif k < 0.7:
            name = f"y{len(iv)}"
            if len(iv) >= 2:
                e = f"{r.choice(iv)} {r.choice(['+', '^', '-', '&'])} {r.choice(iv)}"
            else:
                e = f"ia[(tid + {s}) & 4095]"
            lines.append(f"    int {name} = {e};")
            iv.append(name)
        elif k < 0.9:
            name = f"a{len(av)}"
            base = r.choice(iv) if iv else "tid"
            lines.append(f"    float {name} = fa[({base} + {s}) & 4095];")
            fv.append(name)
            av.append(name)
        else:
            name = f"p{len(pv)}"
            a = r.choice(iv) if iv else "tid"
            lines.append(f"    int {name} = {a} < {r.randint(0, 1000)};")
            iv.append(name)
            pv.append(name)
    fsum = " + ".join(fv[-64:]) if fv else "0.0f"
    isum = " + ".join(iv[-64:]) if iv else "0"
    lines.append(f"    fo[tid] = {fsum};")
    lines.append(f"    io[tid] = {isum};")
    lines.append("}")
    return "\n".join(lines) + "\n"


def regpressure_batch(n: int = 256, seed: int = 4242, n_stmts: int = 6000):
    return [regpressure_kernel(seed + i, i, n_stmts) for i in range(n)]


def pack(srcs):
    """list[str|bytes] -> (buffer bytes, tu_off int64[n+1])."""
    bs = [s.encode() if isinstance(s, str) else bytes(s) for s in srcs]
    off = np.zeros(len(bs) + 1, dtype=np.int64)
    np.cumsum([len(b) for b in bs], out=off[1:])
    return b"".join(bs), off
