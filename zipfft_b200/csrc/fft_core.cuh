// Register-resident mixed-radix FFT building blocks for sm_100a.
//
// The FFTs here replace the cuFFTDx Block FFTs that zipFFT calls in
// src/cuda/real_conv_2d.cuh:26,52,84,114 (forward r2c rows, fused c2c columns,
// inverse c2r rows).  They are written from the textbook Stockham autosort
// formulation (Stockham 1966; Govindaraju et al., SC'08) with FP32 arithmetic on
// the CUDA cores:
//
//   * an N-point transform is split into stages of radix 16, 8, 4, 2, 15, 5 and
//     3 (15 as a prime-factor 3 x 5 butterfly);
//   * every stage runs N/R independent radix-R butterflies held in registers;
//   * stages exchange data through one padded shared-memory buffer;
//   * input and output are both in natural order, so a forward transform's last
//     stage and an inverse transform (run with the radices reversed) share their
//     register layout -- the fused column kernel multiplies by the image spectrum
//     between them without any reordering.
//
// All DFT constants are computed at compile time from the Taylor series of
// sin/cos in double precision (cx_sincos below); twiddle tables are computed on
// the host in double precision and rounded once to float.
#pragma once

#include <cstring>
#include <type_traits>

#if defined(__CUDACC__)
#include <cuda_runtime.h>
#define ZF_HD __host__ __device__ __forceinline__
#define ZF_DEV __device__ __forceinline__
#else
// Host compilation is used only by the CPU test harness of the kernel logic,
// which defines the CUDA keywords before including this header.
#define ZF_HD inline
#define ZF_DEV inline
#endif

namespace zf {

// Order-preserving unsigned key of a float (larger float, larger key; 0 is
// below every float's key), for atomicMax on unsigned words, and its inverse.
ZF_HD unsigned ordered_key(float v) {
    unsigned u;
    memcpy(&u, &v, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
ZF_HD float key_value(unsigned k) {
    const unsigned u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    float v;
    memcpy(&v, &u, 4);
    return v;
}

// ---------------------------------------------------------------------------
// Compile-time trigonometry (double precision Taylor series)
// ---------------------------------------------------------------------------
constexpr double kPi = 3.141592653589793238462643383279502884;

// sin(x) and cos(x) for |x| <= pi by Taylor series (40 terms: error < 1e-18).
constexpr double cx_sin_series(double x) {
    double term = x, sum = x;
    for (int n = 1; n < 40; ++n) {
        term *= -x * x / double((2 * n) * (2 * n + 1));
        sum += term;
    }
    return sum;
}
constexpr double cx_cos_series(double x) {
    double term = 1.0, sum = 1.0;
    for (int n = 1; n < 40; ++n) {
        term *= -x * x / double((2 * n - 1) * (2 * n));
        sum += term;
    }
    return sum;
}
// cos(2 pi m / n) and sin(2 pi m / n) for integers m, n > 0.
constexpr double cx_cos2pi(long m, long n) {
    m %= n;
    if (m < 0) m += n;
    if (2 * m > n) m -= n;  // angle in (-pi, pi]
    return cx_cos_series(2.0 * kPi * double(m) / double(n));
}
constexpr double cx_sin2pi(long m, long n) {
    m %= n;
    if (m < 0) m += n;
    if (2 * m > n) m -= n;
    return cx_sin_series(2.0 * kPi * double(m) / double(n));
}

// ---------------------------------------------------------------------------
// Complex helpers (float2 = {re, im})
//
// The butterflies below are written with lane-wise helpers (px_*) and fold
// every quarter turn (+-i) into a sum or difference (c_add_rot / c_sub_rot),
// so no rotation costs an instruction of its own.  The helpers are scalar
// FP32 operations.  The packed FADD2 / FMUL2 / FFMA2 instructions of sm_100a
// were measured as well (same FP32 lane throughput, half the issue slots; an
// operand may broadcast, swap or negate the halves of its register pair at no
// cost): one B200 ran the 4096^2 / 256^2 step 2.8% slower with them (the
// inverse row pass 36.0 us against 34.6 us per template, the column pass
// unchanged).
// ---------------------------------------------------------------------------
ZF_HD float2 c_make(float re, float im) {
    float2 r;
    r.x = re;
    r.y = im;
    return r;
}
// lane-wise a + b, a * b, a * b + c (round to nearest)
ZF_HD float2 px_add(float2 a, float2 b) { return c_make(a.x + b.x, a.y + b.y); }
ZF_HD float2 px_mul(float2 a, float2 b) { return c_make(a.x * b.x, a.y * b.y); }
ZF_HD float2 px_fma(float2 a, float2 b, float2 c) {
    return c_make(fmaf(a.x, b.x, c.x), fmaf(a.y, b.y, c.y));
}
ZF_HD float2 c_swap(float2 a) { return c_make(a.y, a.x); }
ZF_HD float2 c_add(float2 a, float2 b) { return px_add(a, b); }
ZF_HD float2 c_sub(float2 a, float2 b) { return px_add(a, c_make(-b.x, -b.y)); }
ZF_HD float2 c_neg(float2 a) { return c_make(-a.x, -a.y); }
ZF_HD float2 c_conj(float2 a) { return c_make(a.x, -a.y); }
ZF_HD float2 c_scale(float2 a, float s) { return px_mul(a, c_make(s, s)); }
// a * b, each component with one fused multiply-add.
ZF_HD float2 c_mul(float2 a, float2 b) {
    return c_make(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
// a * conj(b)
ZF_HD float2 c_mul_conj(float2 a, float2 b) {
    return c_make(fmaf(a.x, b.x, a.y * b.y), fmaf(a.y, b.x, -a.x * b.y));
}
// conj(a) * b
ZF_HD float2 c_conj_mul(float2 a, float2 b) {
    return c_make(fmaf(a.x, b.x, a.y * b.y), fmaf(a.x, b.y, -a.y * b.x));
}
// a * (-i) for the forward direction, a * (+i) for the inverse direction.
template <bool INV>
ZF_HD float2 c_rot(float2 a) {
    return INV ? c_make(-a.y, a.x) : c_make(a.y, -a.x);
}
// a * i
ZF_HD float2 c_mul_i(float2 a) { return c_make(-a.y, a.x); }
// t + rot<INV>(d) and t - rot<INV>(d): the swapped d against (+-1, -+1).
template <bool INV>
ZF_HD float2 c_add_rot(float2 t, float2 d) {
    return px_fma(c_swap(d), INV ? c_make(-1.f, 1.f) : c_make(1.f, -1.f), t);
}
template <bool INV>
ZF_HD float2 c_sub_rot(float2 t, float2 d) {
    return px_fma(c_swap(d), INV ? c_make(1.f, -1.f) : c_make(-1.f, 1.f), t);
}
// t + s * rot<INV>(d) for a real constant s.
template <bool INV>
ZF_HD float2 c_add_rot_scaled(float2 t, float2 d, float s) {
    return px_fma(c_swap(d), INV ? c_make(-s, s) : c_make(s, -s), t);
}
// a * (wr + i wi) for constants.
ZF_HD float2 c_mul_const(float2 a, float wr, float wi) {
    return px_fma(c_make(a.x, a.x), c_make(wr, wi), px_mul(c_make(a.y, a.y), c_make(-wi, wr)));
}

// Multiply by the compile-time root of unity exp(-+2 pi i M / N) (forward sign
// "-", inverse sign "+").  Exact special cases avoid multiplications; the
// butterflies below fold quarter turns (+-i) into the following sum instead
// (c_add_rot / c_sub_rot).
template <int M, int N, bool INV>
ZF_HD float2 c_mul_w(float2 a) {
    constexpr int m0 = ((M % N) + N) % N;
    constexpr int m = INV ? (N - m0) % N : m0;  // inverse == forward with -M
    if constexpr (m == 0) {
        return a;
    } else if constexpr (2 * m == N) {
        return c_neg(a);
    } else if constexpr (4 * m == N) {
        return c_make(a.y, -a.x);  // * (-i)
    } else if constexpr (4 * m == 3 * N) {
        return c_make(-a.y, a.x);  // * (+i)
    } else {
        constexpr float wr = float(cx_cos2pi(m, N));
        constexpr float wi = float(-cx_sin2pi(m, N));
        return c_mul_const(a, wr, wi);
    }
}
// True when c_mul_w<M, N, INV> is a quarter turn (then equal to c_rot<Q>
// with Q = quarter_turn_inv<M, N, INV>()).
template <int M, int N, bool INV>
constexpr bool is_quarter_turn() {
    constexpr int m0 = ((M % N) + N) % N;
    constexpr int m = INV ? (N - m0) % N : m0;
    return 4 * m == N || 4 * m == 3 * N;
}
template <int M, int N, bool INV>
constexpr bool quarter_turn_inv() {  // +i (true) or -i (false)
    constexpr int m0 = ((M % N) + N) % N;
    constexpr int m = INV ? (N - m0) % N : m0;
    return 4 * m == 3 * N;
}

// Calls f(std::integral_constant<int, I>) for I = 0 .. N-1 (compile-time index).
template <int N, int I = 0, class F>
ZF_HD void static_for(F&& f) {
    if constexpr (I < N) {
        f(std::integral_constant<int, I>{});
        static_for<N, I + 1>(f);
    }
}

// ---------------------------------------------------------------------------
// Small DFTs in registers: v[0..R) natural order in, natural order out.
// Forward: X[k] = sum_n x[n] exp(-2 pi i n k / R); inverse uses exp(+...),
// unnormalised.
// ---------------------------------------------------------------------------
template <bool INV>
ZF_HD void dft2(float2& a, float2& b) {
    float2 t = a;
    a = c_add(t, b);
    b = c_sub(t, b);
}

// 4-point DFT; with ROT2 the input a2 arrives unrotated and is multiplied by
// rot<INV> (a quarter turn) inside, folded into the first sums.
template <bool INV, bool ROT2 = false>
ZF_HD void dft4(float2& a0, float2& a1, float2& a2, float2& a3) {
    float2 t0, t1;
    if constexpr (ROT2) {
        t0 = c_add_rot<INV>(a0, a2);
        t1 = c_sub_rot<INV>(a0, a2);
    } else {
        t0 = c_add(a0, a2);
        t1 = c_sub(a0, a2);
    }
    const float2 t2 = c_add(a1, a3);
    const float2 t3 = c_sub(a1, a3);
    a0 = c_add(t0, t2);
    a2 = c_sub(t0, t2);
    a1 = c_add_rot<INV>(t1, t3);
    a3 = c_sub_rot<INV>(t1, t3);
}

// 8 = 4 x 2 Cooley-Tukey: DFT4 on even/odd halves, twiddle, DFT2.
template <bool INV>
ZF_HD void dft8(float2* v) {
    dft4<INV>(v[0], v[2], v[4], v[6]);  // E[k1] at v[0],v[2],v[4],v[6]
    dft4<INV>(v[1], v[3], v[5], v[7]);  // O[k1] at v[1],v[3],v[5],v[7]
    v[3] = c_mul_w<1, 8, INV>(v[3]);
    v[7] = c_mul_w<3, 8, INV>(v[7]);
    // X[k1] = E + w O, X[k1+4] = E - w O (w_8^2 = rot<INV>, folded)
    float2 e0 = v[0], e1 = v[2], e2 = v[4], e3 = v[6];
    float2 o0 = v[1], o1 = v[3], o2 = v[5], o3 = v[7];
    v[0] = c_add(e0, o0);
    v[4] = c_sub(e0, o0);
    v[1] = c_add(e1, o1);
    v[5] = c_sub(e1, o1);
    v[2] = c_add_rot<INV>(e2, o2);
    v[6] = c_sub_rot<INV>(e2, o2);
    v[3] = c_add(e3, o3);
    v[7] = c_sub(e3, o3);
}

// 16 = 4 x 4 Cooley-Tukey.
template <bool INV>
ZF_HD void dft16(float2* v) {
    // Step 1: for each n2, DFT4 over x[4 n1 + n2]; result k1 stays in slot 4 k1 + n2.
    dft4<INV>(v[0], v[4], v[8], v[12]);
    dft4<INV>(v[1], v[5], v[9], v[13]);
    dft4<INV>(v[2], v[6], v[10], v[14]);
    dft4<INV>(v[3], v[7], v[11], v[15]);
    // Step 2: twiddle slot (4 k1 + n2) by w16^(n2 k1) (w16^4 = rot<INV> is
    // folded into step 3).
    v[5] = c_mul_w<1, 16, INV>(v[5]);
    v[9] = c_mul_w<2, 16, INV>(v[9]);
    v[13] = c_mul_w<3, 16, INV>(v[13]);
    v[6] = c_mul_w<2, 16, INV>(v[6]);
    v[14] = c_mul_w<6, 16, INV>(v[14]);
    v[7] = c_mul_w<3, 16, INV>(v[7]);
    v[11] = c_mul_w<6, 16, INV>(v[11]);
    v[15] = c_mul_w<9, 16, INV>(v[15]);
    // Step 3: for each k1, DFT4 over n2 (slots 4 k1 + 0..3); output k2 goes to
    // X[k1 + 4 k2].
    dft4<INV>(v[0], v[1], v[2], v[3]);
    dft4<INV>(v[4], v[5], v[6], v[7]);
    dft4<INV, true>(v[8], v[9], v[10], v[11]);
    dft4<INV>(v[12], v[13], v[14], v[15]);
    // Slot 4 k1 + k2 now holds X[k1 + 4 k2]: transpose the 4 x 4 index grid.
    float2 t;
    t = v[1]; v[1] = v[4]; v[4] = t;
    t = v[2]; v[2] = v[8]; v[8] = t;
    t = v[3]; v[3] = v[12]; v[12] = t;
    t = v[6]; v[6] = v[9]; v[9] = t;
    t = v[7]; v[7] = v[13]; v[13] = t;
    t = v[11]; v[11] = v[14]; v[14] = t;
}

template <bool INV>
ZF_HD void dft3(float2* v) {
    constexpr float s3 = 0.86602540378443864676f;  // sin(2 pi / 3)
    const float2 t1 = c_add(v[1], v[2]);
    const float2 t2 = px_fma(t1, c_make(-0.5f, -0.5f), v[0]);
    const float2 d = c_sub(v[1], v[2]);
    // forward: X1 = t2 - i s3 d, X2 = t2 + i s3 d (inverse: signs swapped)
    v[0] = c_add(v[0], t1);
    v[1] = c_add_rot_scaled<INV>(t2, d, s3);
    v[2] = c_add_rot_scaled<INV>(t2, d, -s3);
}

template <bool INV>
ZF_HD void dft5(float2* v) {
    constexpr float c1 = float(cx_cos2pi(1, 5));
    constexpr float c2 = float(cx_cos2pi(2, 5));
    constexpr float s1 = float(cx_sin2pi(1, 5));
    constexpr float s2 = float(cx_sin2pi(2, 5));
    const float2 a0 = v[0];
    const float2 t1 = c_add(v[1], v[4]);
    const float2 t2 = c_add(v[2], v[3]);
    const float2 t3 = c_sub(v[1], v[4]);
    const float2 t4 = c_sub(v[2], v[3]);
    const float2 m1 = px_fma(t1, c_make(c1, c1), px_fma(t2, c_make(c2, c2), a0));
    const float2 m2 = px_fma(t1, c_make(c2, c2), px_fma(t2, c_make(c1, c1), a0));
    const float2 n1 = px_fma(t3, c_make(s1, s1), px_mul(t4, c_make(s2, s2)));
    const float2 n2 = px_fma(t3, c_make(s2, s2), px_mul(t4, c_make(-s1, -s1)));
    // forward: X1 = m1 - i n1, X4 = m1 + i n1, X2 = m2 - i n2, X3 = m2 + i n2
    v[0] = c_add(a0, c_add(t1, t2));
    v[1] = c_add_rot<INV>(m1, n1);
    v[4] = c_sub_rot<INV>(m1, n1);
    v[2] = c_add_rot<INV>(m2, n2);
    v[3] = c_sub_rot<INV>(m2, n2);
}

// 15-point DFT by the prime-factor (Good-Thomas) algorithm, 15 = 3 x 5 with
// coprime factors: the inputs x[(5 n1 + 3 n2) mod 15] form a 3 x 5 array whose
// columns take 3-point and whose rows take 5-point DFTs, with no twiddles in
// between, and X[(10 k1 + 6 k2) mod 15] = Y[k1][k2] (10 = 5 (5^-1 mod 3),
// 6 = 3 (3^-1 mod 5)).
template <bool INV>
ZF_HD void dft15(float2* v) {
    float2 a[3][5];
#pragma unroll
    for (int n1 = 0; n1 < 3; ++n1) {
#pragma unroll
        for (int n2 = 0; n2 < 5; ++n2) a[n1][n2] = v[(5 * n1 + 3 * n2) % 15];
    }
#pragma unroll
    for (int n2 = 0; n2 < 5; ++n2) {
        float2 c[3] = {a[0][n2], a[1][n2], a[2][n2]};
        dft3<INV>(c);
#pragma unroll
        for (int k1 = 0; k1 < 3; ++k1) a[k1][n2] = c[k1];
    }
#pragma unroll
    for (int k1 = 0; k1 < 3; ++k1) dft5<INV>(a[k1]);
#pragma unroll
    for (int k1 = 0; k1 < 3; ++k1) {
#pragma unroll
        for (int k2 = 0; k2 < 5; ++k2) v[(10 * k1 + 6 * k2) % 15] = a[k1][k2];
    }
}

template <int R, bool INV>
ZF_HD void dft(float2* v) {
    static_assert(R == 2 || R == 3 || R == 4 || R == 5 || R == 8 || R == 15 || R == 16, "radix");
    if constexpr (R == 2) {
        dft2<INV>(v[0], v[1]);
    } else if constexpr (R == 3) {
        dft3<INV>(v);
    } else if constexpr (R == 4) {
        dft4<INV>(v[0], v[1], v[2], v[3]);
    } else if constexpr (R == 5) {
        dft5<INV>(v);
    } else if constexpr (R == 8) {
        dft8<INV>(v);
    } else if constexpr (R == 15) {
        dft15<INV>(v);
    } else {
        dft16<INV>(v);
    }
}

// ---------------------------------------------------------------------------
// Stockham plan: N = product of radices, largest first (16s, then the left-over
// power of two, then 15s, 5s and 3s), except that a three-stage plan
// 16 x 16 x r is ordered 16, r, 16.
// ---------------------------------------------------------------------------
struct PlanInfo {
    int S;
    int R[16];
};

constexpr bool fft_size_factorable(int n) {
    if (n < 16) return false;
    while (n % 2 == 0) n /= 2;
    while (n % 3 == 0) n /= 3;
    while (n % 5 == 0) n /= 5;
    return n == 1;
}

constexpr PlanInfo make_plan(int n) {
    PlanInfo p{0, {0}};
    int pow2 = 1;
    while (n % 2 == 0) {
        n /= 2;
        pow2 *= 2;
    }
    while (pow2 >= 16) {
        p.R[p.S++] = 16;
        pow2 /= 16;
    }
    if (pow2 > 1) p.R[p.S++] = pow2;  // 8, 4 or 2
    while (n % 15 == 0) {  // a 3 and a 5 together: one prime-factor radix-15 stage
        p.R[p.S++] = 15;
        n /= 15;
    }
    while (n % 5 == 0) {
        p.R[p.S++] = 5;
        n /= 5;
    }
    while (n % 3 == 0) {
        p.R[p.S++] = 3;
        n /= 3;
    }
    // 16, 16, r -> 16, r, 16 (r = 2, 4, 8 or 15): a palindromic plan, whose
    // reversed inverse shares the forward transform's twiddles (the column
    // pass then holds one twiddle set instead of two).
    if (p.S == 3 && p.R[0] == 16 && p.R[1] == 16) {
        p.R[1] = p.R[2];
        p.R[2] = 16;
    }
    return p;
}

// Padded shared-memory index: one extra float2 every 16 keeps both the
// stride-R writes of the first stage and the unit-stride reads bank-conflict
// free for 64-bit accesses.
ZF_HD int spad(int i) { return i + (i >> 4); }
constexpr int spad_size(int n) { return n + (n >> 4) + 1; }

// One N-point transform executed by T cooperating threads.
//   INV : inverse (exp(+...)) instead of forward
//   REV : radices applied in reverse order
// Stage s has N/R butterflies; thread t owns butterflies b = t + q T.
// Butterfly b of stage s reads elements b + r N/R (r < R) and, after the
// twiddle w_{Ns R}^{(b mod Ns) r} and the radix-R DFT, writes element r to
// (b / Ns) Ns R + (b mod Ns) + r Ns, where Ns is the product of earlier radices.
template <int N, int T, bool INV, bool REV>
struct Stockham {
    static constexpr PlanInfo P = make_plan(N);
    static constexpr int S = P.S;
    static constexpr int kThreads = T;
    static_assert(fft_size_factorable(N), "FFT size must be 2^a 3^b 5^c >= 16");

    static constexpr int radix(int s) { return REV ? P.R[S - 1 - s] : P.R[s]; }
    static constexpr int ns(int s) {
        int p = 1;
        for (int i = 0; i < s; ++i) p *= radix(i);
        return p;
    }
    static constexpr int nbf(int s) { return N / radix(s); }
    static constexpr int bpt(int s) { return (nbf(s) + T - 1) / T; }
    static constexpr int elems(int s) { return bpt(s) * radix(s); }
    static constexpr int max_elems() {
        int m = 0;
        for (int s = 0; s < S; ++s) m = elems(s) > m ? elems(s) : m;
        return m;
    }
    static constexpr int MAXE = max_elems();
    // Number of twiddles a thread needs over stages 1..S-1.
    static constexpr int tw_offset(int s) {
        int o = 0;
        for (int i = 1; i < s; ++i) o += bpt(i) * (radix(i) - 1);
        return o;
    }
    static constexpr int NTW = tw_offset(S) > 0 ? tw_offset(S) : 1;

    // True when every thread owns exactly bpt(s) valid butterflies.
    static constexpr bool even(int s) { return bpt(s) * T == nbf(s); }

    // ---- per-thread twiddle cache ----------------------------------------
    // tw[tw_offset(s) + q (R-1) + r - 1] = w_{Ns R}^{(b mod Ns) r} (forward
    // sign), read from a table of TN-th roots of unity (TN a multiple of N).
    struct Twiddles {
        float2 w[NTW];
        float2 r0[bpt(S > 1 ? 1 : 0)];  // w_{R0}^{b mod R0} for the pruned start
    };

    template <int TN>
    ZF_DEV static void load_twiddles(Twiddles& tw, const float2* __restrict__ table, int t) {
        static_assert(TN % N == 0, "twiddle table must be a multiple of N");
        load_twiddles_stage<1, TN>(tw, table, t);
        if constexpr (S > 1) {
            constexpr int R0 = radix(0);
#pragma unroll
            for (int q = 0; q < bpt(1); ++q) {
                int b = t + q * T;
                tw.r0[q] = __ldg(table + (b % R0) * (TN / R0));
            }
        }
    }
    template <int s, int TN>
    ZF_DEV static void load_twiddles_stage(Twiddles& tw, const float2* __restrict__ table, int t) {
        if constexpr (s < S) {
            constexpr int R = radix(s), NS = ns(s), L = NS * R;
            constexpr int stride = TN / L;
#pragma unroll
            for (int q = 0; q < bpt(s); ++q) {
                int b = t + q * T;
                int bm = b % NS;
                bool ok = even(s) || b < nbf(s);
#pragma unroll
                for (int r = 1; r < R; ++r) {
                    float2 w = c_make(1.f, 0.f);
                    if (ok) w = __ldg(table + bm * r * stride);
                    tw.w[tw_offset(s) + q * (R - 1) + r - 1] = w;
                }
            }
            load_twiddles_stage<s + 1, TN>(tw, table, t);
        }
    }

    // ---- per-thread twiddle tables --------------------------------------
    // A thread's NTW twiddles followed by its NR0 pruned-start roots, in
    // pairs: unit j (float4) of thread t at tab[j * T + t], so that a warp's
    // load of unit j is one contiguous 512-byte request (loading from the
    // shared root table touches up to 32 sectors per request, at every
    // launch).  fill_thread_twiddles builds a thread's units with
    // load_twiddles itself, so the values are the same.
    static constexpr int NR0 = bpt(S > 1 ? 1 : 0);
    static constexpr int TWU = (NTW + NR0 + 1) / 2;
    ZF_HD static float2 tw_get(const Twiddles& tw, int k) {
        return k < NTW ? tw.w[k] : tw.r0[k - NTW];
    }
    ZF_HD static void tw_set(Twiddles& tw, int k, float2 v) {
        if (k < NTW)
            tw.w[k] = v;
        else
            tw.r0[k - NTW] = v;
    }
    template <int TN>
    ZF_DEV static void fill_thread_twiddles(float4* tab, const float2* __restrict__ table, int t) {
        Twiddles tw;
        load_twiddles<TN>(tw, table, t);
        for (int j = 0; j < TWU; ++j) {
            const float2 a = tw_get(tw, 2 * j);
            const float2 b = 2 * j + 1 < NTW + NR0 ? tw_get(tw, 2 * j + 1) : c_make(0.f, 0.f);
            float4 u;
            u.x = a.x;
            u.y = a.y;
            u.z = b.x;
            u.w = b.y;
            tab[j * T + t] = u;
        }
    }
    ZF_DEV static void load_thread_twiddles(Twiddles& tw, const float4* __restrict__ tab, int t) {
#pragma unroll
        for (int j = 0; j < TWU; ++j) {
            const float4 u = __ldg(tab + j * T + t);
            tw_set(tw, 2 * j, c_make(u.x, u.y));
            if (2 * j + 1 < NTW + NR0) tw_set(tw, 2 * j + 1, c_make(u.z, u.w));
        }
    }

    // ---- stage primitives -------------------------------------------------
    // Butterflies of stage s on registers v (twiddle first, then DFT).
    template <int s, class TWS>
    ZF_DEV static void compute(float2 (&v)[MAXE], const TWS& tw) {
        constexpr int R = radix(s);
#pragma unroll
        for (int q = 0; q < bpt(s); ++q) {
            if constexpr (s > 0) {
#pragma unroll
                for (int r = 1; r < R; ++r) {
                    float2 w = tw.w[tw_offset(s) + q * (R - 1) + r - 1];
                    v[q * R + r] = INV ? c_mul_conj(v[q * R + r], w) : c_mul(v[q * R + r], w);
                }
            }
            dft<R, INV>(&v[q * R]);
        }
    }

    // Offsets of element r within a butterfly fold into one padded base when
    // the element stride is a multiple of 16 (spad(x + r*S) = spad(x) + r*spad(S)),
    // or when the whole butterfly lies inside one 16-element block.
    static constexpr bool load_folds(int s) { return nbf(s) % 16 == 0; }
    static constexpr bool store_folds(int s) {
        return ns(s) % 16 == 0 || (16 % (ns(s) * radix(s)) == 0);
    }
    static constexpr int store_off(int s) { return ns(s) % 16 == 0 ? ns(s) + ns(s) / 16 : ns(s); }

    // Read the inputs of stage s from the shared buffer.
    template <int s>
    ZF_DEV static void load(float2 (&v)[MAXE], const float2* buf, int t) {
        constexpr int R = radix(s), NB = nbf(s);
#pragma unroll
        for (int q = 0; q < bpt(s); ++q) {
            const int b = t + q * T;
            if (even(s) || b < NB) {
                if constexpr (load_folds(s)) {
                    const float2* p = buf + spad(b);
#pragma unroll
                    for (int r = 0; r < R; ++r) v[q * R + r] = p[r * (NB + NB / 16)];
                } else {
#pragma unroll
                    for (int r = 0; r < R; ++r) v[q * R + r] = buf[spad(b + r * NB)];
                }
            }
        }
    }

    // Write the outputs of stage s to the shared buffer.
    template <int s>
    ZF_DEV static void store(const float2 (&v)[MAXE], float2* buf, int t) {
        constexpr int R = radix(s), NB = nbf(s), NS = ns(s);
#pragma unroll
        for (int q = 0; q < bpt(s); ++q) {
            const int b = t + q * T;
            if (even(s) || b < NB) {
                const int base = (b / NS) * NS * R + (b % NS);
                if constexpr (store_folds(s)) {
                    float2* p = buf + spad(base);
#pragma unroll
                    for (int r = 0; r < R; ++r) p[r * store_off(s)] = v[q * R + r];
                } else {
#pragma unroll
                    for (int r = 0; r < R; ++r) buf[spad(base + r * NS)] = v[q * R + r];
                }
            }
        }
    }

    // Stages s .. S-1 where stage s-1's outputs are in registers.  Ends with
    // the last stage's outputs in registers: v[q R + r] = X[b + r N/R].
    // Every thread of the block must call this (it synchronises the block).
    // TAIL = false leaves out the barrier after the last stage's loads; the
    // caller then passes a block barrier of its own before writing buf again.
    template <int s, bool TAIL = true, class TWS>
    ZF_DEV static void run_from(float2 (&v)[MAXE], float2* buf, const TWS& tw, int t) {
        if constexpr (s < S) {
            store<s - 1>(v, buf, t);
            __syncthreads();
            load<s>(v, buf, t);
            if constexpr (TAIL || s + 1 < S) __syncthreads();
            compute<s>(v, tw);
            run_from<s + 1, TAIL>(v, buf, tw, t);
        }
    }

    // Full transform whose stage-0 input is in registers (layout of stage 0).
    template <bool TAIL = true, class TWS>
    ZF_DEV static void run_regs(float2 (&v)[MAXE], float2* buf, const TWS& tw, int t) {
        compute<0>(v, tw);
        run_from<1, TAIL>(v, buf, tw, t);
    }

    // Full transform whose input is in the shared buffer (natural order,
    // padded).  The caller synchronises before the call.
    template <class TWS>
    ZF_DEV static void run_smem(float2 (&v)[MAXE], float2* buf, const TWS& tw, int t) {
        load<0>(v, buf, t);
        __syncthreads();
        compute<0>(v, tw);
        run_from<1>(v, buf, tw, t);
    }

    // Stage at which a transform of a zero-padded input starts computing: 1
    // when stage 0 folds into the reads of stage 1 (NZ in {1, 2}), else 0.
    template <int NZ>
    static constexpr int first_stage() {
        return ((NZ == 1 || NZ == 2) && S >= 2) ? 1 : 0;
    }

    // Inputs of stage first_stage<NZ>() of a forward transform of a
    // zero-padded input given by a loader ld(i) -> x[i] (the loader returns
    // zero past the signal end).  NZ is the number of possibly non-zero
    // inputs per stage-0 butterfly (0 = unknown): for NZ in {1, 2} stage 0 is
    // folded into the reads of stage 1, so the padded region is neither read
    // nor transformed.
    template <int NZ, class LD, class TWS>
    ZF_DEV static void load_input(float2 (&v)[MAXE], const LD& ld, const TWS& tw, int t) {
        constexpr int R0 = radix(0), NB0 = nbf(0);
        if constexpr (first_stage<NZ>() == 1) {
            // Stage-1 input i equals stage-0 output (butterfly m = i / R0,
            // element k = i % R0) = sum_{j < NZ} x[m + j NB0] w_R0^{j k}.
            // Since R0 divides N/R1, k = b mod R0 for every element of
            // butterfly b, so one root per butterfly serves all its elements.
            constexpr int R1 = radix(1), NB1 = nbf(1);
#pragma unroll
            for (int q = 0; q < bpt(1); ++q) {
                int b = t + q * T;
                if (even(1) || b < NB1) {
                    float2 w = tw.r0[q];
                    if (INV) w = c_conj(w);
#pragma unroll
                    for (int r = 0; r < R1; ++r) {
                        int m = (b + r * NB1) / R0;
                        float2 acc = ld(m);
                        if constexpr (NZ == 2) acc = c_add(acc, c_mul(ld(m + NB0), w));
                        v[q * R1 + r] = acc;
                    }
                }
            }
        } else {
#pragma unroll
            for (int q = 0; q < bpt(0); ++q) {
                int b = t + q * T;
                if (even(0) || b < NB0) {
#pragma unroll
                    for (int r = 0; r < R0; ++r) v[q * R0 + r] = ld(b + r * NB0);
                }
            }
        }
    }

    // Full forward transform of a zero-padded input given by a loader (see
    // load_input).  The twiddle set TWS is this transform's Twiddles, or that
    // of a transform with the same radix sequence (a palindromic plan run in
    // reverse).  TAIL as in run_from.
    template <int NZ, bool TAIL = true, class LD, class TWS>
    ZF_DEV static void run_loader(float2 (&v)[MAXE], const LD& ld, float2* buf, const TWS& tw,
                                  int t) {
        load_input<NZ>(v, ld, tw, t);
        if constexpr (first_stage<NZ>() == 1) {
            compute<1>(v, tw);
            run_from<2, TAIL>(v, buf, tw, t);
        } else {
            run_regs<TAIL>(v, buf, tw, t);
        }
    }
};

}  // namespace zf
