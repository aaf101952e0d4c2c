"""Shared helpers for the test modules."""
from __future__ import annotations

import gzip
import json
import random
from functools import lru_cache
from pathlib import Path

GOLDEN = Path(__file__).resolve().parent / "golden"


@lru_cache(maxsize=None)
def golden(name: str):
    with gzip.open(GOLDEN / name, "rt", encoding="utf-8") as f:
        return json.load(f)


RAISE_CODE = {"ValueError": 1, "OverflowError": 2}


def check_digests(gold, idx, texts, statuses):
    """Compare engine results with a golden digest record
    (``oracle/goldens.py``): TU ``idx[j]`` of the workload gave status
    ``statuses[j]`` and text ``texts[j]`` (bytes or str; ignored unless the
    status is 0).  Every TU must be byte-identical, or raise where the
    reference raises (same exception class); returns the count of each."""
    import hashlib
    n_ok = n_raise = 0
    for j, i in enumerate(idx):
        st, gs = int(statuses[j]), int(gold["status"][i])
        if gs != 0:
            assert st == gs, (i, "reference raises", gs, "engine status", st)
            n_raise += 1
            continue
        assert st == 0, (i, "engine status", st)
        t = texts[j]
        b = t.encode("utf-8", "surrogateescape") if isinstance(t, str) else bytes(t)
        assert hashlib.sha256(b).digest() == bytes(gold["digest"][i]), (i, "PTX differs")
        n_ok += 1
    return n_ok, n_raise


def fuzz_sources(n: int, seed: int, maxlen: int = 80):
    r = random.Random(seed)
    alpha = list("\"'/*\\\n \t\r.0123456789xXeEpP+-fFuUlLabz_=<>&|!;#@\x0c") + [
        "0x1.8p3", "1e+", "'\\n'", "/*", "*/", "//", '"a\\"b"', "0x", "..",
        "1.e5f", "0x.p1", "0x1p1024", "0x1.fffffffffffff8p1023", "int", "for"]
    return ["".join(r.choice(alpha) for _ in range(r.randint(0, maxlen))) for _ in range(n)]


PP_NAMES = ['A', 'B', 'AB', 'F', 'G', 'FG', 'X_1', 'defined', 'N']


def pp_fuzz_sources(n: int, seed: int):
    """Seeded directive-heavy TUs for the preprocessor (no macro whose body
    calls itself: the reference never returns on those)."""
    r = random.Random(seed)
    out = []
    for _ in range(n):
        lines = []
        for _ in range(r.randint(1, 25)):
            k = r.random()
            nm = r.choice(PP_NAMES)
            if k < 0.15:
                lines.append(f"#define {nm} " + r.choice(
                    ['1', 'A + B', '(x)', 'F(1, 2)', 'AB*2', '', 'B', '0x10u', 'A // c', '"s"',
                     'x\\ty', 'q\\n']))
            elif k < 0.25:
                body = r.choice(['a + b', '(a)*2', 'a ## b', '__VA_ARGS__', 'f(a, b)', 'a',
                                 'G(a)', 'x', 'F(a)', 'AB(b)'])
                if body.startswith(nm + '('):
                    body = 'a'
                params = r.choice(['a', 'a, b', 'x, ...', '', ' a , b '])
                lines.append(f"#define {nm}({params}) {body}")
            elif k < 0.30:
                lines.append(f"#undef {nm}")
            elif k < 0.36:
                lines.append(f"#ifdef {nm}")
            elif k < 0.40:
                lines.append(f"#ifndef {nm}")
            elif k < 0.45:
                lines.append("#if " + r.choice(
                    ['1', '0', 'A', 'defined(A)', 'defined B', 'A == 1', 'A && B', '!A',
                     'A + 1 > 2', '1 < 2 < 3', '(A)', '2**3 == 8', '7 // 2 == 3', '1 << 4',
                     'FG', '', '-7 % 3 == 2', '0x1F & 3', '1/0', '3 > 2 > 1']))
            elif k < 0.48:
                lines.append('#elif A')
            elif k < 0.53:
                lines.append(r.choice(['#else', '#endif', '# endif', '#endif // x', '  #  else']))
            elif k < 0.56:
                lines.append(r.choice(['#include "x.h"', '#include <y.h>', '# include "a b"',
                                       '#pragma once', '#line 5', '#error no']))
            elif k < 0.60:
                lines.append(r.choice(['x = A + \\', '  B;', 'y \\', '\\']))
            else:
                lines.append(r.choice(['x = A + B;', 'F(1, 2);', 'FG(A, (B, 3));', 'G(F(1,2))',
                                       'AB = A*B', 's = "A";', 'N(1)', 'F (x)', 'call(F,G)',
                                       'y = AB + FG;', 'defined', 'F("a\\n")', 'G(\'q\')']))
        out.append("\n".join(lines) + r.choice(["", "\n"]))
    return out


# Hand-written kernels covering the parser's constructs (and its error paths);
# the expected IR always comes from the reference itself.
PARSE_CASES = [
    # control flow: while / do / break / continue / nested loops
    """__global__ void k(int *a, int n) {
    int i = threadIdx.x; int s = 0;
    while (i < n) { s += a[i]; if (s > 100) break; i += blockDim.x; }
    do { s--; if (s & 1) continue; s = s >> 1; } while (s > 10);
    for (int j = 0; j < 4; j++) for (int q = j; q < 4; ++q) { s ^= q * j; }
    a[threadIdx.x] = s;
}""",
    # ternary, && and || with side effects in the rhs
    """__global__ void k(float *x, int *y, int n) {
    int t = blockIdx.x * blockDim.x + threadIdx.x;
    int v = 0;
    float f = t < n ? x[t] : 0.0f;
    if (t < n && (v = y[t]) != 0) f += 1.0f;
    if (t >= n || y[t] == 3) f -= 2.0f;
    int m = (t > 5) ? t : -t;
    x[t] = f * m + v;
}""",
    # casts, sizeof, unsigned / long long literals, shifts, ~ and !
    """__global__ void k(unsigned int *o, long long *p, const float * __restrict__ in) {
    unsigned int u = 0xFFFFFFFFu;
    long long q = 123456789012LL;
    int b = (int)in[threadIdx.x];
    float c = (float)b / 3;
    unsigned long long z = (unsigned long long)u << 3;
    o[0] = u >> 4; o[1] = ~u; o[2] = !b; o[3] = sizeof(float) + sizeof(double*);
    p[0] = q * 2 + z; p[1] = (long long)c;
    o[4] = 017 + 0x1F + 10u + 'a' + '\\n';
}""",
    # shared arrays (1D, 2D, scalar, extern), __syncthreads, 2D indexing
    """__global__ void k(float *out) {
    __shared__ float tile[16][17];
    __shared__ int cnt;
    extern __shared__ float dyn[];
    __shared__ float a[32], b[64];
    int tx = threadIdx.x, ty = threadIdx.y;
    tile[ty][tx] = out[ty * 16 + tx];
    if (tx == 0) cnt = 0;
    __syncthreads();
    a[tx] = tile[tx][ty] + dyn[tx];
    b[tx] = a[tx] * 2.0f + cnt;
    out[ty * 16 + tx] = b[tx];
}""",
    # local arrays with aggregate initializers, compound stores, ++ on elements
    """__global__ void k(int *o) {
    int w[4] = {1, 2, 3, 4};
    int m[2][3] = {{1, 2, 3}, {4, 5, 6}};
    float acc[8];
    w[1] += 5; w[2]++; w[3] <<= 1;
    acc[threadIdx.x & 7] = 1.5f;
    o[threadIdx.x] = w[threadIdx.x & 3] + m[1][2] + (int)acc[0];
}""",
    # pointer arithmetic, pointer variables, *p stores, p++ / p += n
    """__global__ void k(float *base, int n) {
    float *p = base + threadIdx.x;
    float *q = p;
    *p = 1.0f;
    p++;
    p += 2;
    *p = *q + 3.0f;
    q = q - 1;
    q[0] = p[1];
    float *r = &base[4];
    *r += 2.0f;
}""",
    # intrinsics: shuffles, ballot, atomics, __ldg, math, min/max, warpSize
    """__global__ void k(float *x, int *c, unsigned int *m) {
    float v = __ldg(&x[threadIdx.x]);
    v += __shfl_down_sync(0xffffffff, v, 16);
    v = fmaxf(v, 0.0f) + sqrtf(fabsf(v)) + expf(v) + __fmaf_rn(v, v, 1.0f);
    unsigned int b = __ballot_sync(0xffffffffu, v > 1.0f);
    int pc = __popc(b) + __clz(b) + min(threadIdx.x, 3u) + max(1, 2) + warpSize;
    atomicAdd(&c[0], pc);
    atomicMax(&c[1], pc);
    atomicCAS(&c[2], 0, 1);
    m[threadIdx.x] = b + __any_sync(0xffffffff, pc > 3) + __all_sync(0xffffffff, pc);
    __threadfence();
    __syncwarp();
    x[threadIdx.x] = v;
}""",
    # half and double types, typedef'd ints, launch bounds, multiple kernels
    """__global__ void __launch_bounds__(256, 2) k1(double *d, int64_t *e, size_t n) {
    double a = d[0] * 2.0;
    uint32_t u = 7;
    e[0] = (int64_t)a + u + n;
}
__global__ void k2(half *h, bool flag) {
    half x = h[0];
    if (flag) h[1] = x;
}""",
    # scoping: shadowing in blocks, for-init scope, labels, goto, empty statements
    """__global__ void k(int *a) {
    int x = a[0];
    { int x = 5; a[1] = x; }
    for (int x = 0; x < 3; x++) { a[2] += x; }
    ;;
    lbl: a[3] = x;
    goto lbl;
    if (x) { int y = x * 2; x = y; } else { int y = 3; x -= y; }
    a[4] = x;
}""",
    # module-level consts, __shared__ and templates, static, namespace, forward decl
    """const int N = 64;
static const float SCALE = 0.5f;
__shared__ float gsh[128];
__global__ void fwd(int *a);
namespace ns {
template <typename T>
__global__ void k(float *o, int *a) {
    gsh[threadIdx.x] = o[threadIdx.x] * SCALE;
    a[threadIdx.x % N] = N;
}
}""",
    # comma expressions, compound assignment chains, assignment in conditions
    """__global__ void k(int *a, int n) {
    int i, j = 1, k2;
    i = 0, j = 2;
    for (i = 0, k2 = n; i < k2; i += 2, k2--) { a[i] = k2; }
    int t = (j = 5, j + 1);
    a[0] = t; a[1] = j;
    a[2] = (a[3] = 7);
    int u = 3; u *= u += 2;
    a[4] = u;
}""",
    # volatile, const qualifiers, unsigned char/short, signed types, enum type
    """__global__ void k(volatile int *flag, const unsigned char *b, short *s, unsigned short *us) {
    volatile __shared__ int v;
    signed char c = b[0];
    unsigned short w = us[0];
    enum E e = 0;
    long int li = 3;
    signed long long sl = -1;
    v = c + w + li + sl + e;
    flag[0] = v;
    s[0] = (short)v;
}""",
    # float constant folding and literal forms
    """__global__ void k(float *o) {
    float a = 1.5f * 2.0f + 3.25e-2f - .5f + 1.f;
    float b = 10 / 4 + 10 % 3 - (-7) / 2 + (-7) % 2;
    double c = 1e10 * 3.0;
    int d = (1 << 4) | (0xF0 >> 2) ^ 3 & 7;
    o[0] = a + b + c + d;
    o[1] = 1.0f / 0.0f;
}""",
    # parse errors (the reference raises ParseError)
    """__global__ void k(int *a) { a[0] = ; }""",
    """__global__ void k(int *a) { int x = undefined_var + 1; a[0] = x; }""",
    """__global__ void k(int *a) { break; }""",
    """__global__ void k(int *a) { a[0] = 1 }""",
    """__global__ void k(int *a { }""",
    # ValueError from int() of a malformed literal
    """__global__ void k(int *a) { a[0] = 09; }""",
    # unterminated kernel body (IndexError / ParseError at EOF)
    """__global__ void k(int *a) { a[0] = 1;""",
    # no kernels at all
    """int x; float y;""",
    "",
    # template-parameter type heuristic: (N) casts, (N + 1) parses as an expression
    """__global__ void k(float *o, int N) {
    o[0] = (N) * 2;
    o[1] = (N + 1);
    o[2] = (T)3;
}""",
    # return statements with and without values, code after return
    """__global__ void k(int *a, int n) {
    if (n < 0) return;
    a[0] = n;
    return;
    a[1] = 2;
}""",
    # pointer-to-pointer indexing and casts between address spaces
    """__global__ void k(float **rows, int r, int c) {
    rows[r][c] = 1.0f;
    float *row = rows[r];
    row[c + 1] = rows[0][0];
    float *g = (float *)row;
    g[0] = 2.0f;
}""",
    # nested ternary / logical mixes inside loops with loop-carried values
    """__global__ void k(int *a, int n) {
    int s = 0, p = 1;
    for (int i = 0; i < n; i++) {
        s = (i & 1) ? s + i : s - i;
        p = (p > 100 || s < 0) ? 1 : p * 2;
        if (s > 10 && p < 50) { s -= p; continue; }
        a[i] = s + p;
    }
    a[n] = s;
}""",
]


def mutate_sources(n: int, seed: int):
    """Seeded token-level mutations (delete / insert / replace) of the hand
    cases and of generated kernels: inputs for the parser's error paths."""
    import re
    from opencuda import synth
    r = random.Random(seed)
    base = PARSE_CASES + synth.random_batch(50, seed=seed)
    toks_re = re.compile(r"\s+|[A-Za-z_]\w*|\d+\.?\d*[fFuUlL]*|\S")
    extra = ['(', ')', '{', '}', ';', ',', '*', '&', '[', ']', '=', '+', '?', ':', 'int',
             'float', 'if', 'for', 'while', 'x', 'N', '0', '1.0f', '&&', '||', '++', '--',
             'return', 'break', '__shared__', 'unsigned', 'T', 'sizeof', '->', '.', '<<', '!']
    out = []
    for _ in range(n):
        t = toks_re.findall(r.choice(base))
        for _ in range(r.randint(1, 3)):
            if not t:
                break
            j = r.randrange(len(t))
            op = r.random()
            if op < 0.4:
                del t[j]
            elif op < 0.7:
                t.insert(j, ' ' + r.choice(extra) + ' ')
            else:
                t[j] = ' ' + r.choice(extra) + ' '
        out.append(''.join(t))
    return out


SWITCH_CASES = [
    # plain cases with breaks, default last
    """__global__ void s0(int *o, int n) {
    int t = threadIdx.x; int r = 0;
    switch (t & 3) {
    case 0: r = 10; break;
    case 1: r = n * 2; break;
    case 2: r = r + 5; break;
    default: r = -1; break;
    }
    o[t] = r;
}""",
    # fallthrough chains, default in the middle, empty cases
    """__global__ void s1(float *o, int k) {
    int t = threadIdx.x; float a = 1.0f; int c = 0;
    switch (k) {
    case 1:
    case 2: a = a * 2.0f;
    case 3: a = a + 1.0f; c = c + 1; break;
    default: a = 0.5f;
    case 7: c = c + 7;
    }
    o[t] = a + c;
}""",
    # no default, switch on an expression, an empty switch
    """__global__ void s2(int *o, int *in) {
    int t = threadIdx.x; int v = in[t]; int acc = v;
    switch (v * 3 + 1) { case 4: acc = acc + 1; break; case 7: acc = acc ^ 5; }
    switch (t) { }
    o[t] = acc;
}""",
    # switch in a loop: break leaves the switch, continue the loop
    """__global__ void s3(int *o, int n) {
    int t = threadIdx.x; int s = 0;
    for (int i = 0; i < n; i++) {
        switch (i & 3) {
        case 0: s = s + i; break;
        case 1: continue;
        case 2: s = s * 2; if (s > 100) { s = 0; break; } s = s + 1; break;
        default: s = s - 1;
        }
        s = s + 3;
    }
    o[t] = s;
}""",
    # nested switches and a loop inside a case, constant-folded switch value
    """__global__ void s4(float *o, int a, int b) {
    int t = threadIdx.x; float f = 0.0f; int m = 4;
    switch (a) {
    case 0:
        switch (b) { case 0: f = 1.0f; break; case 1: f = 2.0f; break; default: f = 3.0f; }
        break;
    case 1:
        for (int j = 0; j < 4; j++) { f = f + j; }
        break;
    default:
        while (m > 0) { m = m - 1; f = f * 1.5f; }
    }
    switch (2) { case 2: f = f + 0.25f; break; default: f = -f; }
    o[t] = f;
}""",
    # declarations inside cases, unsigned and char case labels
    """__global__ void s5(unsigned *o, unsigned u) {
    int t = threadIdx.x; unsigned r = 0;
    switch (u) {
    case 0u: { unsigned q = u + 9u; r = q * 2u; break; }
    case 'a': r = 97u;
    case 0x10: r = r + 16u; break;
    }
    o[t] = r;
}""",
    # break outside a loop or switch -> ParseError in the reference
    """__global__ void s6(int *o) { int t = threadIdx.x; switch (t) { case 0: o[t] = 1; } break; }""",
    # default only, and a return inside a case
    """__global__ void s7(int *o, int k) {
    int t = threadIdx.x;
    switch (k) { default: o[t] = 3; }
    switch (k) { case 5: return; case 6: o[t] = 6; }
    o[t] = o[t] + 1;
}""",
]


def switch_sources(n: int, seed: int):
    """Seeded random kernels built around switch statements: nested
    switch/if/for, fallthrough, break/continue, defaults anywhere."""
    r = random.Random(seed)
    out = []
    for i in range(n):
        ints = ["a", "b", "c"]
        lines = [f"__global__ void sw{i}(int *o, int *in, int n) {{",
                 "    int t = threadIdx.x;", "    int a = in[t]; int b = n; int c = 1;"]

        def stmt(depth, in_loop, in_sw):
            k = r.random()
            v, w = r.choice(ints), r.choice(ints)
            if depth < 3 and k < 0.3:
                lab = r.sample(range(-2, 12), r.randint(0, 4))
                body = [f"switch ({v} {r.choice(['&', '%', '+'])} {r.randint(1, 5)}) {{"]
                dpos = r.randint(0, len(lab)) if r.random() < 0.6 else -1
                for j in range(len(lab) + 1):
                    if j == dpos:
                        body.append("default:")
                    elif j < len(lab):
                        body.append(f"case {lab[j]}:")
                    else:
                        continue
                    for _ in range(r.randint(0, 2)):
                        body.extend(stmt(depth + 1, in_loop, True))
                    if r.random() < 0.6:
                        body.append("break;")
                body.append("}")
                return body
            if depth < 3 and k < 0.4:
                return [f"for (int i{depth} = 0; i{depth} < {r.randint(1, 5)}; i{depth}++) {{",
                        *stmt(depth + 1, True, in_sw), "}"]
            if depth < 3 and k < 0.5:
                return [f"if ({v} > {w}) {{", *stmt(depth + 1, in_loop, in_sw), "} else {",
                        *stmt(depth + 1, in_loop, in_sw), "}"]
            if in_loop and k < 0.55:
                return ["continue;"]
            if (in_loop or in_sw) and k < 0.6:
                return ["break;"]
            return [f"{v} = {w} {r.choice(['+', '-', '*', '^'])} {r.randint(0, 9)};"]

        for _ in range(r.randint(1, 4)):
            lines.extend("    " + s for s in stmt(0, False, False))
        lines.append("    o[t] = a + b * c;")
        lines.append("}")
        out.append("\n".join(lines) + "\n")
    return out


TYPEDEF_ENUM_CASES = [
    # enum constants with implicit and explicit values, a tag used as a type
    """enum Mode { M_ADD, M_MUL = 4, M_SUB, M_LAST = M_SUB + 10 };
__global__ void e0(int *o, int k) {
    int t = threadIdx.x; enum Mode m = M_MUL; Mode q = (Mode)k;
    int r = (k == M_ADD) ? t + M_LAST : t * M_SUB;
    o[t] = r + m + q;
}""",
    # anonymous enum, trailing comma, float and negative initializers
    """enum { A0 = -3, A1, A2 = 2.75, A3, };
__global__ void e1(float *o) { int t = threadIdx.x; o[t] = A0 + A1 * A2 - A3; }""",
    # scalar and pointer typedefs, typedef of a typedef, unsigned aliases
    """typedef float real;
typedef unsigned int u32;
typedef real *realp;
typedef u32 word;
__global__ void e2(realp out, const real *in, word n) {
    u32 t = threadIdx.x; real s = 0.0f;
    for (word i = 0; i < 4; i++) { s = s + in[(t + i) & 63]; }
    if (t < n) out[t] = s * (real)2;
}""",
    # typedef enum with an alias, used in a switch; enum defined after the kernel
    """typedef enum { RED, GREEN = 5, BLUE } Color;
__global__ void e3(int *o, int k) {
    int t = threadIdx.x; Color c = (Color)k; int v = 0;
    switch (c) { case RED: v = LATE_A; break; case GREEN: v = 2; break; case BLUE: v = 3; break; default: v = -1; }
    o[t] = v + LATE_B;
}
enum { LATE_A = 11, LATE_B };""",
    # array typedef (dimension dropped), function-pointer typedef, redefinition
    """typedef float vec8[8];
typedef int (*binop)(int, int);
typedef int T1;
typedef double T1;
__global__ void e4(float *o, T1 d) { int t = threadIdx.x; vec8 x = 1.5f; T1 y = d * 2.0; o[t] = x + y; }""",
    # a typedef name shadowing a builtin typedef, sizeof of typedefs
    """typedef long long int64_t;
typedef unsigned char byte;
__global__ void e5(unsigned long long *o) {
    int t = threadIdx.x; int64_t a = t; byte b = 200;
    o[t] = a * sizeof(int64_t) + sizeof(byte) + b;
}""",
    # errors: a typedef without a name, an enumerator that is not an identifier
    """typedef float;\n__global__ void e6(float *o) { o[0] = 1.0f; }""",
    """enum { 3, B };\n__global__ void e7(int *o) { o[0] = 1; }""",
    # an enum that is never closed
    """enum E { P, Q\n__global__ void e8(int *o) { o[0] = P; }""",
]


def typedef_enum_sources(n: int, seed: int):
    """Seeded kernels that declare enums (tags, explicit and implicit values)
    and scalar/pointer typedefs at module scope and use them in declarations,
    casts and arithmetic."""
    r = random.Random(seed)
    scal = ["int", "unsigned int", "float", "double", "long long", "unsigned char", "short"]
    out = []
    for i in range(n):
        lines, consts, types = [], [], []
        for e in range(r.randint(1, 3)):
            names = [f"K{i}_{e}_{j}" for j in range(r.randint(1, 5))]
            parts = []
            for nm in names:
                if consts and r.random() < 0.3:
                    parts.append(f"{nm} = {r.choice(consts)} + {r.randint(0, 9)}")
                elif r.random() < 0.3:
                    parts.append(f"{nm} = {r.randint(-20, 40)}")
                else:
                    parts.append(nm)
                consts.append(nm)
            tag = f"Tag{e}" if r.random() < 0.5 else ""
            if tag:
                types.append(f"enum {tag}" if r.random() < 0.5 else tag)
            lines.append(f"enum {tag} {{ {', '.join(parts)} }};")
        for d in range(r.randint(1, 3)):
            base = r.choice(scal + [t for t in types if not t.startswith("enum")])
            alias = f"ty{d}"
            lines.append(f"typedef {base} {alias};")
            types.append(alias)
        body = ["    int t = threadIdx.x;"]
        vars_ = ["t"]
        for s in range(r.randint(2, 8)):
            ty = r.choice(types + ["int", "float"])
            e1 = r.choice(consts + vars_)
            e2 = r.choice(consts + vars_)
            expr = f"({ty})({e1} {r.choice(['+', '-', '*'])} {e2})"
            body.append(f"    {ty} v{s} = {expr};")
            vars_.append(f"v{s}")
        body.append(f"    o[t] = {' + '.join(vars_[-4:])};")
        lines.append(f"__global__ void te{i}(float *o) {{")
        lines.extend(body)
        lines.append("}")
        out.append("\n".join(lines) + "\n")
    return out


DEVFUNC_CASES = [
    # scalar helper with one return
    """__device__ float sq(float x) { return x * x; }
__global__ void d0(float *o, const float *in) { int t = threadIdx.x; o[t] = sq(in[t]) + sq(2.0f); }""",
    # several returns, called in a loop and in a condition
    """__device__ int clampi(int v, int lo, int hi) {
    if (v < lo) return lo;
    if (v > hi) return hi;
    return v;
}
__global__ void d1(int *o, int n) {
    int t = threadIdx.x; int s = 0;
    for (int i = 0; i < 8; i++) { s = s + clampi(t - i, 0, n); }
    if (clampi(s, 0, 100) > 50) s = s * 2;
    o[t] = s;
}""",
    # void helper writing through a pointer, early `return;`
    """__device__ void put(float *p, int i, float v) {
    if (i < 0) return;
    p[i] = v * 0.5f;
}
__global__ void d2(float *o, int n) { int t = threadIdx.x; put(o, t - 3, 1.0f); put(o, n, 2.0f); }""",
    # nested calls, callee defined after the caller, qualifiers and a prototype
    """__device__ float g(float x);
__device__ __forceinline__ float f(float a, float b) { return g(a) * b + g(b); }
static __device__ float g(float x) { return x + 1.0f; }
__global__ void d3(float *o, float k) { int t = threadIdx.x; o[t] = f(f(k, 2.0f), g(k)); }""",
    # locals named like the caller's, a loop inside the helper, threadIdx inside
    """__device__ int acc(int n) {
    int s = 0;
    for (int i = 0; i < n; i++) { s = s + i * threadIdx.x; }
    return s;
}
__global__ void d4(int *o) {
    int s = 7; int i = 3;
    int r = acc(4) + acc(i);
    o[threadIdx.x] = r + s + i;
}""",
    # double and unsigned helpers, a helper used in a switch and a ternary
    """__device__ double lerp(double a, double b, double t) { return a + (b - a) * t; }
__device__ unsigned mix(unsigned x) { return (x ^ (x >> 3)) * 2654435761u; }
__global__ void d5(double *o, unsigned k) {
    int t = threadIdx.x; double v = 0.0;
    switch (mix(k) & 3u) { case 0: v = lerp(1.0, 2.0, 0.25); break; default: v = lerp(0.0, 8.0, 0.5); }
    o[t] = (mix(t) > 100u) ? v : -v;
}""",
    # a helper that only declares, and one returning a pointer
    """__device__ void nothing(int x) { int y = x + 1; }
__device__ float *at(float *p, int i) { return p + i; }
__global__ void d6(float *o) { int t = threadIdx.x; nothing(t); *at(o, t) = 3.0f; }""",
]

# recursive __device__ functions: the reference emits .func bodies for them
DEVFUNC_RECURSIVE_CASES = [
    """__device__ int fact(int n) { if (n <= 1) return 1; return n * fact(n - 1); }
__global__ void r0(int *o) { o[threadIdx.x] = fact(threadIdx.x & 7); }""",
    """__device__ int ping(int n);
__device__ int pong(int n) { return n <= 0 ? 0 : ping(n - 1) + 1; }
__device__ int ping(int n) { return n <= 0 ? 0 : pong(n - 1) + 2; }
__global__ void r1(int *o) { o[threadIdx.x] = ping(5); }""",
]


def devfunc_sources(n: int, seed: int):
    """Seeded kernels calling chains of small scalar __device__ helpers
    (several returns, loops, nested calls, helpers defined before or after
    their callers)."""
    r = random.Random(seed)
    out = []
    for i in range(n):
        nf = r.randint(1, 4)
        funcs = []
        for j in range(nf):
            ty = r.choice(["int", "float", "unsigned int"])
            name = f"h{i}_{j}"
            body = [f"__device__ {ty} {name}({ty} a, {ty} b) {{"]
            body.append(f"    {ty} c = a {r.choice(['+', '-', '*'])} b;")
            if r.random() < 0.5:
                body.append(f"    if (c > ({ty}){r.randint(0, 50)}) return c {r.choice(['+', '*'])} a;")
            if r.random() < 0.4:
                body.append(f"    for (int k = 0; k < {r.randint(1, 4)}; k++) {{ c = c + ({ty})k; }}")
            if j > 0 and r.random() < 0.6:
                callee = funcs[r.randrange(j)][0]
                body.append(f"    c = c + ({ty}){callee}(({funcs[r.randrange(j)][1]})a, "
                            f"({funcs[r.randrange(j)][1]})b);")
            body.append(f"    return c {r.choice(['+', '-', '^'] if ty != 'float' else ['+', '-'])} b;")
            body.append("}")
            funcs.append((name, ty, "\n".join(body)))
        order = funcs[:]
        if r.random() < 0.3:  # define callees after callers, with prototypes first
            protos = [f"__device__ {ty} {nm}({ty} a, {ty} b);" for nm, ty, _ in funcs]
            text = "\n".join(protos) + "\n" + "\n".join(b for _, _, b in reversed(order))
        else:
            text = "\n".join(b for _, _, b in order)
        calls = []
        for k in range(r.randint(1, 4)):
            nm, ty, _ = r.choice(funcs)
            calls.append(f"    {ty} v{k} = {nm}(({ty})(t + {k}), ({ty})in[t & 63]);")
        kern = [f"__global__ void dk{i}(float *o, const int *in) {{", "    int t = threadIdx.x;",
                *calls, f"    o[t] = {' + '.join(f'(float)v{k}' for k in range(len(calls)))};", "}"]
        out.append(text + "\n" + "\n".join(kern) + "\n")
    return out


ADDR_OF_CASES = [
    # out-parameters through device helpers, reloaded after the call
    """__device__ void divmod(int a, int b, int *q, int *r) { *q = a / b; *r = a - (a / b) * b; }
__global__ void a0(int *o, int n) {
    int t = threadIdx.x; int q = 0; int r = 0;
    divmod(t + n, 7, &q, &r);
    o[t] = q * 10 + r;
}""",
    # the same variable spilled twice, read through the pointer, a float slot
    """__device__ void bump(float *p, float d) { *p = *p + d; }
__global__ void a1(float *o) {
    int t = threadIdx.x; float acc = 1.0f;
    bump(&acc, 2.0f);
    bump(&acc, (float)t);
    float *pa = &acc;
    o[t] = acc + *pa;
}""",
    # &x without a call: later reads keep the old value, writes go to the slot
    """__global__ void a2(int *o) {
    int t = threadIdx.x; int x = t * 3;
    int *p = &x;
    *p = 5;
    o[t] = x + *p;
}""",
    # &(expression) spills the value of the expression
    """__device__ int twice(int *p) { return *p * 2; }
__global__ void a3(int *o, int k) { int t = threadIdx.x; o[t] = twice(&k) + twice(&t); }""",
    # & in a loop and in a branch
    """__device__ void inc(int *p) { *p = *p + 1; }
__global__ void a4(int *o, int n) {
    int t = threadIdx.x; int c = 0;
    for (int i = 0; i < 4; i++) { if (i < n) inc(&c); }
    o[t] = c;
}""",
]


# calls the reference's emitter has no case for: no instruction is emitted,
# only the destination register is taken
UNKNOWN_CALL_CASES = [
    """__global__ void u0(float *o, const float *in) {
    int t = threadIdx.x; float x = in[t];
    float a = __expf(x); float b = __fdividef(x, 3.0f); float c = __saturatef(x);
    o[t] = a + b + c + sqrtf(x);
}""",
    """__global__ void u1(int *o, int k) {
    int t = threadIdx.x;
    int p = __builtin_popcount(k); int q = my_helper(t, k);
    o[t] = p * q + t;
}""",
    """__global__ void u2(double *o, double d) { int t = threadIdx.x; o[t] = __dadd_rn(d, 1.0) + sin(d); }""",
]

INTRINSIC_CASES = [
    """__global__ void i0(float *o, const float *in) {
    int t = threadIdx.x; float x = in[t]; float y = in[t + 1];
    o[t] = powf(x, y) + hypotf(x, 2.0f) + cbrtf(y) + powf(x, 2.0f);
}""",
    """__global__ void i1(int *o, unsigned *u, int k) {
    int t = threadIdx.x;
    o[t] = __mul24(t, k) + __mulhi(t, 123456789) + (int)__umulhi(u[t], 77u) + (int)__umul24(u[t], 3u);
    u[t] = __byte_perm(u[t], u[t + 1], 0x3210) + __byte_perm(u[t], 0u, 0x0123);
}""",
]

CAST_CASES = [
    """__global__ void c0(float *o, const int *in, unsigned char *b) {
    int t = threadIdx.x;
    float f = static_cast<float>(in[t]);
    int i = static_cast<int>(f * 2.5f);
    unsigned u = reinterpret_cast<unsigned>(i);
    float *p = const_cast<float *>(o);
    p[t] = f + static_cast<double>(u) + static_cast<float>(b[t]);
}""",
    """__global__ void c1(int *o) {
    __shared__ float s[32];
    int t = threadIdx.x;
    float *ps = static_cast<float *>(s);
    ps[t] = 1.0f;
    o[t] = static_cast<int>(ps[t]) + static_cast<long long>(t);
}""",
    # an unknown type is not consumed: the '>' is missing (ParseError)
    """__global__ void c2(int *o) { int t = threadIdx.x; o[t] = static_cast<Unknown>(t); }""",
]

HEXFLOAT_CASES = [
    """__global__ void h0(float *o, double *d) {
    int t = threadIdx.x;
    float a = 0x1.8p3f; float b = 0x.8p-2F; float c = 0x10p0;
    d[t] = 0x1.fffffffffffffp1023 * 0.0 + 0x1p-1074 + 0x1.921fb54442d18p+1L;
    o[t] = a * b + c + 0xAp-4;
}""",
]

ARRAY_PARAM_CASES = [
    """__device__ float sum3(float v[3]) { return v[0] + v[1] + v[2]; }
__global__ void ap0(float out[], const float in[256], int n) {
    int t = threadIdx.x;
    float *q = out + 1;
    out[t] = in[t] * 2.0f + sum3(out);
    if (t < n) q[t] = in[t & 255];
}""",
    """__global__ void ap1(int a[], int *b, int k) { int t = threadIdx.x; a[t] = b[t] + a[t + k]; b[t] = a[0]; }""",
]

MORE_INTRINSIC_CASES = [
    """__global__ void m0(float *o, const float *in, int *io, unsigned *u) {
    int t = threadIdx.x; float x = in[t]; float y = in[t + 1];
    o[t] = atan2f(y, x) + atanf(x) + atan2f(1.0f, y);
    io[t] = __dp4a(io[t], io[t + 1], 7) + (int)__dp4a_u(u[t], 3u, 1u);
    u[t] = __funnelshift_l(u[t], u[t + 1], 5) + __funnelshift_rc(u[t], 0u, (unsigned)t);
}""",
]

HALF_REDUCE_CASES = [
    """__global__ void h0(__half *o, const __half *a, const __half *b, float *f, int n) {
    int t = threadIdx.x;
    __half x = a[t]; __half y = b[t];
    __half s = __hadd(x, y); __half m = __hmul(s, y); __half d = __hsub(m, x);
    __half q = __hdiv(d, y); __half r = __hfma(x, y, q);
    o[t] = __hmax(__habs(r), __hneg(__hmin(x, y)));
    f[t] = __half2float(r) + __low2float(__hsqrt(x)) + __half2float(__hexp(y)) + __half2float(__hlog10(x));
    f[t + n] = (float)(__hlt(x, y) + __hisnan(r) + __heq(s, m));
    o[t + n] = __float2half(f[t]) ;
    o[t + 2 * n] = __float2half_rz(f[t + n]);
}""",
    """__global__ void h1(unsigned short *u, __half *o, int *io) {
    int t = threadIdx.x;
    __half h = __ushort_as_half(u[t]);
    u[t + 1] = __half_as_ushort(h);
    o[t] = __int2half_rn(io[t]);
    io[t] = __half2int_rz(h) + __hadd(io[t], t) + __rhadd(t, 3);
    o[t + 1] = __hceil(h);
}""",
    """__global__ void r0(int *o, const int *a, unsigned *u, float *f) {
    int t = threadIdx.x;
    int v = a[t];
    o[t] = __reduce_add_sync(0xffffffff, v) + __reduce_min_sync(0xffffffff, v) + __reduce_max_sync(0xffffffff, v);
    u[t] = __reduce_and_sync(0xffffffffu, u[t]) ^ __reduce_or_sync(0xffffffffu, u[t]) ^ __reduce_xor_sync(0xffffffffu, u[t])
         ^ __reduce_umin_sync(0xffffffffu, u[t]) ^ __reduce_umax_sync(0xffffffffu, u[t]);
    o[t + 32] = __match_any_sync(0xffffffff, v);
    f[t] = asinf(f[t]) + acosf(f[t + 1]);
}""",
]

GLOBAL_VAR_CASES = [
    """__device__ int g_counter;
__device__ float g_scale = 2.0f;
__device__ int g_table[16];
__global__ void k(int *out, float *f, const int *idx, int n) {
    int t = threadIdx.x;
    if (t < n) {
        out[t] = atomicAdd(&g_counter, 1);
        f[t] = f[t] * g_scale;
        int i = idx[t] & 15;
        out[t + n] = g_table[i] + atomicAdd(&g_table[i], 2);
    }
}""",
    """__device__ __constant__ int dc_int = 100;
__constant__ __device__ float cd_float = 2.5f;
__constant__ float c_only = 1.5f;
__constant__ __device__ int cd_table[8] = {1, 2, 3, 4, 5, 6, 7, 8};
__constant__ double c_d[4] = {1.0, 2.0, 3.0, 4.0};
__global__ void c(float *out, int *io, double *d, int n) {
    int tid = threadIdx.x;
    if (tid < n) {
        out[tid] = (float)dc_int * cd_float + c_only * (float)tid;
        io[tid] = cd_table[io[tid] & 7] * tid;
        d[tid] = c_d[tid & 3] + c_d[0];
    }
}""",
    """__device__ float g_acc;
__device__ int g_hist[32];
__device__ volatile int g_flag;
__device__ unsigned long long g_big;
__device__ char g_c[7];
__device__ short g_s;
__global__ void w(const float *in, int n) {
    int t = threadIdx.x + blockIdx.x * blockDim.x;
    g_acc = in[t];
    g_acc += 1.0f;
    g_hist[t & 31] = t;
    g_hist[t & 31] += n;
    g_hist[(t + 1) & 31] -= g_hist[t & 31];
    g_flag = 1;
    while (g_flag == 0) { }
    g_big = (unsigned long long)t * 3ull;
    g_c[t & 3] = (char)t;
    g_s = (short)n;
    for (int i = 0; i < 4; ++i) g_hist[i] = g_hist[i] + i;
}""",
    """__global__ void after(float *o, int n) {
    int t = threadIdx.x;
    if (t < n) o[t] = late_w[t & 3] * late_s;
}
__device__ float late_w[4] = {0.25f, 0.25f, 0.25f, 0.25f};
__constant__ float late_s = 3.0f;
__device__ float *g_ptr;
__global__ void ptrs(float *o) {
    int t = threadIdx.x;
    g_ptr = o;
    o[t] = (float)t;
}""",
]

GLOBAL_2D_CASES = [
    """__device__ float g_m[4][8];
__device__ double g_d[3][5];
__global__ void m1(float *o, int n) {
    int t = threadIdx.x;
    g_m[t & 3][t & 7] = (float)t;
    g_m[1][2] += 1.0f;
    g_d[n][t] = 0.5;
    o[t] = (float)t;
}""",
    """__device__ float g_m[4][8];
__device__ int g_c[2][3][4];
__global__ void m2(float *o, int n) {
    int t = threadIdx.x;
    g_m[t & 3][t & 7] = (float)t;
    g_m[1][2] += 1.0f;
    g_c[1][t & 3][0] = n;
    o[t] = g_m[t & 3][0] + (float)g_c[0][1][2];
}""",
    """__constant__ float c_k[3][3] = {{1, 2, 1}, {2, 4, 2}, {1, 2, 1}};
__constant__ int c_after = 5;
__global__ void cv(float *o, const float *in, int w) {
    int t = threadIdx.x;
    o[t] = in[t] * c_k[1][1] + (float)c_after;
}""",
]


# struct / union / vector-type kernels (parser.py:98-128, :3876-3942 and the
# StructTy paths of the expression, statement and kernel parsers)
STRUCT_CASES = [
    # local struct: zero-initialized fields, field stores and reads
    """struct Acc { float sum; int count; };
__global__ void s0(float *o, const float *in, int n) {
    struct Acc a;
    a.sum = 0.5f; a.count = n;
    a.sum = a.sum + in[threadIdx.x];
    a.count += 2;
    o[threadIdx.x] = a.sum * (float)a.count;
}""",
    # aggregate initializer (an int literal into a float field is retyped)
    """typedef struct { float x, y, z; } P3;
__global__ void s1(float *o) {
    P3 p = {1, 2.5f, threadIdx.x};
    o[threadIdx.x] = p.x + p.y * p.z;
}""",
    # pointer to struct: element fields loaded, stored, through -> and [i].
    """struct Particle { float px, py; float vx, vy; int alive; };
__global__ void s2(struct Particle *ps, float dt, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        if (ps[i].alive) {
            ps[i].px = ps[i].px + ps[i].vx * dt;
            ps[i].py += ps[i].vy * dt;
        }
        struct Particle *q = &ps[i];
        q->vy = q->vy - 9.8f * dt;
    }
}""",
    # struct by value as a kernel parameter (one .param per field)
    """struct Cfg { int n; float scale; float *dst; };
__global__ void s3(struct Cfg c, const float *src) {
    int i = threadIdx.x;
    if (i < c.n) c.dst[i] = src[i] * c.scale;
}""",
    # device functions taking and returning structs, several returns
    """struct V2 { float x; float y; };
__device__ struct V2 add2(struct V2 a, struct V2 b) { struct V2 r; r.x = a.x + b.x; r.y = a.y + b.y; return r; }
__device__ struct V2 pick(struct V2 a, struct V2 b, int k) { if (k > 0) return a; return b; }
__global__ void s4(float *o, int k) {
    struct V2 a = {1.0f, 2.0f};
    struct V2 b; b.x = (float)threadIdx.x; b.y = 3.0f;
    struct V2 c = add2(a, b);
    struct V2 d = pick(c, a, k);
    o[threadIdx.x] = c.x * d.y + d.x;
}""",
    # struct fields carried around a loop (write-back of the field values)
    """struct St { int lo; int hi; float w; };
__global__ void s5(float *o, const int *in, int n) {
    struct St s; s.lo = 0; s.hi = 0; s.w = 1.0f;
    for (int i = 0; i < n; i++) {
        if (in[i] < 0) s.lo = s.lo + 1; else s.hi = s.hi + in[i];
        s.w = s.w * 0.5f;
    }
    o[threadIdx.x] = (float)(s.hi - s.lo) * s.w;
}""",
    # CUDA vector types
    """__global__ void s6(float *o, int *oi) {
    float3 a; a.x = 1.0f; a.y = 2.0f; a.z = (float)threadIdx.x;
    float4 b = {a.x, a.y, a.z, 4.0f};
    int2 c; c.x = threadIdx.x; c.y = c.x * 2;
    double2 d; d.x = 1.5; d.y = (double)b.w;
    uint4 u; u.w = 7u;
    o[threadIdx.x] = a.x + b.y * b.w + (float)d.y;
    oi[threadIdx.x] = c.x + c.y + (int)u.w;
}""",
    # union, anonymous typedef'd struct, nested struct fields
    """union Bits { float f; unsigned int u; };
struct Inner { int a; int b; };
typedef struct { float m; struct Inner in; } Outer;
struct Box { float lo[3]; float hi[3]; };
__global__ void s7(float *o, Outer *po, struct Box *bx) {
    union Bits v; v.f = 2.0f; v.u = v.u + 1u;
    Outer q = po[threadIdx.x];
    float e = bx[0].hi[1] - bx[0].lo[1];
    o[threadIdx.x] = v.f + q.m + (float)(q.in.a) + e;
}""",
    # array members: constant and run-time indices, through pointer and value
    """struct Hist { int bins[4]; float total; };
__global__ void s8(struct Hist *h, int *o, int k) {
    struct Hist l;
    l.bins[2] = 5; l.total = 1.0f;
    h->bins[k & 3] = l.bins[2];
    o[threadIdx.x] = h->bins[1] + l.bins[6];
}""",
    # an array member through an element lvalue: KeyError in the reference
    """struct Hist { int bins[4]; };
__global__ void s8b(struct Hist *h) { h[1].bins[2] = 9; }""",
    # module variables of struct type, a __constant__ struct array
    """struct Par { float a; float b; int n; };
__device__ struct Par g_par;
__constant__ struct Par c_tab[4];
__global__ void s9(float *o) {
    int t = threadIdx.x;
    g_par.a = 3.0f;
    o[t] = c_tab[t & 3].b + (float)c_tab[1].n;
}""",
    # __shared__ and local arrays of structs
    """struct Cell { float v; int id; };
__global__ void s10(float *o, int n) {
    __shared__ struct Cell tile[64];
    struct Cell loc[4];
    int t = threadIdx.x;
    tile[t].v = (float)t; tile[t].id = t;
    loc[t & 3].v = 2.0f;
    __syncthreads();
    o[t] = tile[(t + 1) & 63].v + loc[1].v + (float)tile[t].id;
}""",
    # &struct passed to a helper that writes through the pointer
    """struct Pair { int a; int b; };
__device__ void swap_pair(struct Pair *p) { int t = p->a; p->a = p->b; p->b = t; }
__global__ void s11(int *o) {
    struct Pair p; p.a = threadIdx.x; p.b = 7;
    swap_pair(&p);
    o[threadIdx.x] = p.a * 10 + p.b;
}""",
    # compound literals, struct copies, struct stores through a pointer
    """typedef struct { float x; float y; } Vec2;
__device__ Vec2 mk(float a, float b) { return (Vec2){a, b}; }
__global__ void s12(Vec2 *out, float s) {
    Vec2 a = mk(s, 2.0f);
    Vec2 b;
    b = a;
    b.y = b.y * s;
    out[threadIdx.x] = b;
    *out = a;
}""",
    # sizeof of struct types, pointer arithmetic over structs
    """struct Rec { double d; int i; char c; };
__global__ void s13(int *o, struct Rec *r) {
    struct Rec *p = r + 2;
    p++;
    o[threadIdx.x] = sizeof(struct Rec) + sizeof(float4) + (int)p->i;
}""",
    # a field the struct does not have: KeyError in the reference
    """struct A { int x; };
__global__ void s14(int *o) { struct A a; a.x = 1; o[0] = a.y; }""",
    # an undefined struct: ParseError
    """__global__ void s15(int *o) { struct Missing m; o[0] = 1; }""",
    # struct defined after the kernel that uses it (module pass 1)
    """__global__ void s16(float *o) { struct Late l; l.v = 2.0f; o[threadIdx.x] = l.v; }
struct Late { float v; };""",
]


def struct_sources(n: int, seed: int):
    """Seeded kernels over random struct types: mixed scalar, pointer, array
    and nested fields; locals with and without initializers, field updates in
    branches and loops, element access through struct pointers, structs passed
    to and returned from device helpers, and vector types."""
    r = random.Random(seed)
    scal = ["int", "float", "unsigned int", "double", "long long"]
    out = []
    for i in range(n):
        nf = r.randint(2, 5)
        fields = []
        for j in range(nf):
            k = r.random()
            if k < 0.7:
                fields.append((r.choice(scal), f"f{j}", 0))
            elif k < 0.85:
                fields.append((r.choice(["int", "float"]), f"a{j}", r.randint(2, 4)))
            else:
                fields.append(("float *", f"p{j}", 0))
        sname = f"S{i}"
        decl = " ".join(f"{t} {nm}[{c}];" if c else f"{t} {nm};" for t, nm, c in fields)
        text = [f"struct {sname} {{ {decl} }};"]
        scal_f = [(t, nm) for t, nm, c in fields if not c and "*" not in t]
        arr_f = [(t, nm, c) for t, nm, c in fields if c]
        if not scal_f:
            scal_f = [("int", "fz")]
            text[0] = f"struct {sname} {{ {decl} int fz; }};"
        use_fn = r.random() < 0.5
        if use_fn:
            t0, n0 = r.choice(scal_f)
            text.append(f"__device__ struct {sname} upd{i}(struct {sname} s, {t0} v) {{")
            text.append(f"    s.{n0} = s.{n0} + v;")
            if r.random() < 0.5:
                text.append(f"    if (v > ({t0})3) return s;")
            text.append(f"    s.{n0} = s.{n0} * ({t0})2;")
            text.append("    return s;")
            text.append("}")
        vec = r.choice(["float2", "float3", "float4", "int2", "int4", "uint2", "double2"])
        body = [f"__global__ void st{i}(struct {sname} *ps, float *o, int n) {{",
                "    int t = threadIdx.x;",
                f"    struct {sname} a;"]
        for t, nm in scal_f:
            if r.random() < 0.7:
                body.append(f"    a.{nm} = ({t})(t + {r.randint(0, 9)});")
        if r.random() < 0.5:
            body.append(f"    struct {sname} b = ps[t & 15];")
        else:
            body.append(f"    struct {sname} b; b = a;")
        t0, n0 = r.choice(scal_f)
        if r.random() < 0.6:
            body.append(f"    for (int k = 0; k < {r.randint(2, 8)}; k++) {{")
            body.append(f"        if (k < n) a.{n0} = a.{n0} + ({t0})k; else b.{n0} = b.{n0} - ({t0})1;")
            body.append("    }")
        if arr_f:
            t1, n1, c1 = r.choice(arr_f)
            body.append(f"    a.{n1}[{r.randint(0, c1 - 1)}] = ({t1})t;")
            body.append(f"    ps[t].{n1}[n & {c1 - 1 if c1 in (2, 4) else 1}] = a.{n1}[{r.randint(0, c1 - 1)}];")
        if use_fn:
            body.append(f"    struct {sname} c = upd{i}(a, ({t0})n);")
        else:
            body.append(f"    struct {sname} c = a;")
        body.append(f"    ps[t].{n0} = c.{n0} + b.{n0};")
        body.append(f"    {vec} v; v.x = ({ 'double' if vec == 'double2' else 'float' })c.{n0}; v.y = v.x + 1;")
        terms = [f"(float)c.{nm}" for _, nm in scal_f] + ["(float)v.y", f"(float)ps[n].{n0}"]
        body.append(f"    o[t] = {' + '.join(terms)};")
        body.append("}")
        out.append("\n".join(text + body) + "\n")
    return out


# printf, inline asm and the texture / surface / mbarrier intrinsics
# (parser.py:1645-1679, :1732-1738, :2326-2375; codegen/emit.py:1151-1168,
# :1661-1740, :1919-1999)
PRINTF_ASM_CASES = [
    # printf with no argument, int / unsigned / float / double / pointer / 64-bit
    """__global__ void p0(const float *a, int n) {
    int t = threadIdx.x;
    printf("start\\n");
    printf("t=%d u=%u f=%f d=%f p=%p l=%lld\\n", t, (unsigned int)n, a[t], (double)a[t], a, (long long)t);
}""",
    # printf in a branch and in a loop (unrolled), escapes in the format
    """__global__ void p1(int *o, int n) {
    int t = threadIdx.x;
    if (t == 0) printf("tab\\there \\"q\\" back\\\\slash %d\\r\\n", n);
    for (int i = 0; i < 3; i++) printf("i=%d\\n", i + t);
    o[t] = n;
}""",
    # two kernels with printf: one vprintf declaration, per-kernel labels
    """__global__ void pa(int x) { printf("a %d\\n", x); }
__global__ void pb(int x, float y) { printf("b %d %f\\n", x, y); printf("b2\\n"); }""",
    # a string argument: the last string literal becomes the format
    """__global__ void p2(int x) { printf("%s=%d\\n", "x", x); }""",
    # inline PTX with outputs and inputs, volatile, clobbers, several statements
    """__global__ void p3(unsigned int *o, unsigned int a, unsigned int b) {
    unsigned int lane, r;
    asm volatile("mov.u32 %0, %%laneid;" : "=r"(lane));
    asm("add.u32 %0, %1, %2; add.u32 %0, %0, 1;" : "=r"(r) : "r"(a), "r"(b) : "memory");
    o[threadIdx.x] = r + lane;
}""",
    # asm output into a fresh name; empty template emits nothing
    """__global__ void p4(int *o) {
    __asm__("mov.u32 %0, %%tid.x;" : "=r"(fresh));
    asm volatile("" ::: "memory");
    o[0] = fresh;
}""",
    # texture, surface and mbarrier intrinsics (PTX text only)
    """__global__ void p5(float *o, unsigned long long tex, unsigned long long surf, int n) {
    int t = threadIdx.x;
    float a = tex1Dfetch(tex, t);
    float b = tex2D(tex, 0.5f, 1.5f);
    float c = tex3D(tex, 0.5f, 1.5f, 2.5f);
    int s = surf1Dread(surf, t * 4);
    surf1Dwrite(s + 1, surf, t * 4);
    __shared__ unsigned long long bar[1];
    if (t == 0) __mbarrier_init(bar, 32);
    __syncthreads();
    int ok = __mbarrier_try_wait_parity(bar, 0);
    o[t] = a + b + c + (float)ok;
}""",
]


def printf_sources(n: int, seed: int):
    """Seeded kernels with printf calls of random argument mixes inside
    branches and loops, and inline asm adds."""
    r = random.Random(seed)
    out = []
    tys = [("int", "%d"), ("unsigned int", "%u"), ("float", "%f"), ("double", "%f"),
           ("long long", "%lld")]
    for i in range(n):
        body = [f"__global__ void pf{i}(float *o, const int *in, int n) {{",
                "    int t = threadIdx.x;", "    float acc = (float)in[t & 7];"]
        for k in range(r.randint(1, 4)):
            args = [r.choice(tys) for _ in range(r.randint(0, 5))]
            fmt = " ".join(f"v{j}={f}" for j, (_, f) in enumerate(args)) + "\\n"
            vals = [f"({ty})(acc + {j})" for j, (ty, _) in enumerate(args)]
            call = f'printf("k{k} {fmt}"{"".join(", " + v for v in vals)});'
            c = r.random()
            if c < 0.3:
                body.append(f"    if (t < n) {call}")
            elif c < 0.5:
                body.append(f"    for (int i = 0; i < {r.randint(2, 4)}; i++) {{ acc = acc + 1.0f; {call} }}")
            else:
                body.append(f"    {call}")
            if r.random() < 0.3:
                body.append('    int q; asm("add.s32 %0, %1, %2;" : "=r"(q) : "r"(t), "r"(n));')
                body.append("    acc = acc + (float)q;")
        body.append("    o[t] = acc;")
        body.append("}")
        out.append("\n".join(body) + "\n")
    return out


# recursive __device__ functions compiled as .func (parser.py:4089-4153,
# :4392-4435; codegen/emit.py:506-646, :1744-1776, :3126-3154)
RECURSIVE_CASES = [
    """__device__ int fact(int n) { if (n <= 1) return 1; return n * fact(n - 1); }
__global__ void r0(int *o) { o[threadIdx.x] = fact(threadIdx.x & 7); }""",
    # mutual recursion through a prototype
    """__device__ int ping(int n);
__device__ int pong(int n) { return n <= 0 ? 0 : ping(n - 1) + 1; }
__device__ int ping(int n) { return n <= 0 ? 0 : pong(n - 1) + 2; }
__global__ void r1(int *o) { o[threadIdx.x] = ping(5); }""",
    # float and pointer parameters, a void recursive function, a loop inside
    """__device__ float powr(float x, int e) { if (e == 0) return 1.0f; return x * powr(x, e - 1); }
__device__ void fill(float *p, int n, float v) { if (n <= 0) return; p[n - 1] = v; fill(p, n - 1, v * 0.5f); }
__device__ int sum_to(int n) { int s = 0; for (int i = 0; i < 4; i++) s += i; if (n > 0) s += sum_to(n - 1); return s; }
__global__ void r2(float *o, int k) {
    o[threadIdx.x] = powr(1.5f, k);
    fill(o + 32, 8, 1.0f);
    o[64 + threadIdx.x] = (float)sum_to(k);
}""",
    # a non-recursive helper calling a recursive one (inlined at its call)
    """__device__ int fib(int n) { if (n < 2) return n; return fib(n - 1) + fib(n - 2); }
__device__ int twice_fib(int n) { return 2 * fib(n); }
__global__ void r3(int *o, int n) { o[threadIdx.x] = twice_fib(n) + fib(3); }""",
]


def recursive_sources(n: int, seed: int):
    """Seeded modules of 1-6 __device__ functions with random call graphs
    (self calls, mutual cycles, chains into cycles) and names of random
    lengths, called from a kernel."""
    r = random.Random(seed)
    out = []
    alpha = "abcdefghijklmnopqrstuvwxyz_"
    for i in range(n):
        k = r.randint(1, 6)
        names = []
        while len(names) < k:
            nm = r.choice("abcdefghijklmnopqrstuvwxyz") + "".join(
                r.choice(alpha + "0123456789") for _ in range(r.randint(0, 17)))
            if nm not in names:
                names.append(nm)
        tys = [r.choice(["int", "float", "unsigned int"]) for _ in range(k)]
        edges = [sorted(set(r.randrange(k) for _ in range(r.randint(0, 3)))) for _ in range(k)]
        protos = [f"__device__ {tys[j]} {names[j]}(int n);" for j in range(k)]
        defs = []
        for j in range(k):
            terms = [f"({tys[j]}){names[c]}(n - {r.randint(1, 3)})" for c in edges[j]]
            body = " + ".join(terms) if terms else f"({tys[j]})n"
            defs.append(f"__device__ {tys[j]} {names[j]}(int n) {{ if (n <= 0) return ({tys[j]})1; "
                        f"return {body}; }}")
        order = list(range(k))
        r.shuffle(order)
        calls = " + ".join(f"(float){names[j]}(t & {r.randint(1, 7)})"
                           for j in r.sample(range(k), r.randint(1, k)))
        text = "\n".join(protos) + "\n" + "\n".join(defs[j] for j in order) + \
            f"\n__global__ void rk{i}(float *o) {{ int t = threadIdx.x; o[t] = {calls}; }}\n"
        out.append(text)
    return out
