// The three kernels of the implicitly zero-padded real 2D FFT cross-correlation
// (zipFFT: src/cuda/real_conv_2d.cuh:6-117, I/O layer src/cuda/real_conv_2d_io.hpp).
//
// Per template, with image size H x W, template h x w and W2 = W/2:
//
//   k_row_r2c   rows n < h:  X_n = rfft_W(pad(t_n)) * 1/(H W)      (cuh:8-30)
//               written as R[kx][n] (column-major, packed kx = 0..W2-1)
//   k_col_fused columns kx:  Q[.,kx] = IFFT_H( conj(FFT_H(pad_h(R[kx]))) . S[kx] )
//                                                                   (cuh:58-117)
//   k_row_c2r   rows y:      out[y] = irfft_W(Q[y, .])              (cuh:34-56)
//
// Layout of the per-template workspace slice (complex64, column pitch H):
//   element (kx, y) at kx * H + y, packed kx in [0, W2).  Packed column 0
//   holds the two real columns kx = 0 (real part) and kx = W2 (imaginary part).
//   R occupies rows [0, h) of every column; the column kernel replaces it in
//   place by Q, one column per transform, so no two blocks touch the same
//   column.  The slice needs H * W2 complex values, less than the
//   H * (W/2 + 1) the reference's workspace holds per template
//   (real_conv_2d_binding.cu:235-245).
//
// Differences from the reference's layout (real_conv_2d_io.hpp:134-195): the
// reference keeps the workspace row-major and reads it down columns at stride
// W/2+1; here the column kernel reads and writes whole contiguous columns and
// the row kernels move 4 rows at a time so each column segment they touch is
// one 32-byte sector.
//
// The normalisations 1/H (io.hpp:278-282) and 1/W (io.hpp:302-306) are folded
// into the template rows (k_row_r2c), so the column and row-inverse kernels do
// no scaling.
#pragma once

#include "fft_core.cuh"

namespace zf {

#if defined(__CUDACC__)
ZF_DEV float2* dyn_smem() {
    extern __shared__ __align__(16) float2 zf_dyn_smem_arr[];
    return zf_dyn_smem_arr;
}
#else
float2* dyn_smem();  // provided by the CPU test harness
#endif

// Threads per transform: 16 elements per thread in radix-16 stages.
constexpr int fft_threads(int n) { return (n + 15) / 16; }

template <int H>
struct ColCfg {
    static constexpr int T = fft_threads(H);
    static constexpr int FPB = T >= 256 ? 1 : 256 / T;  // columns per block
    static constexpr int THREADS = FPB * T;
    static constexpr int BUF = spad_size(H);  // float2 per column buffer
    static constexpr int SMEM = FPB * BUF * 8;
};

template <int W2>
struct RowCfg {
    static constexpr int T = fft_threads(W2);
    static constexpr int RPB = (256 / T) > 4 ? 256 / T : 4;  // rows per block
    static constexpr int THREADS = RPB * T;
    static constexpr int BUF = spad_size(W2);
    static constexpr int SMEM = RPB * BUF * 8;
};

// True when the radix sequence of n reads the same backwards.  The column
// kernel's inverse runs the radices in reverse, so for such plans it can use
// the forward twiddles (conjugated by the inverse butterflies).
constexpr bool plan_palindrome(int n) {
    PlanInfo p = make_plan(n);
    for (int s = 0; s < p.S; ++s)
        if (p.R[s] != p.R[p.S - 1 - s]) return false;
    return true;
}

// ---------------------------------------------------------------------------
// Loaders: the implicit zero padding (io.hpp:69-100, :134-166).  Indices past
// the signal end return zero without a memory access.
// ---------------------------------------------------------------------------

// Column input: h complex rows of one packed column.  mode 0: the complex
// column; mode 1 / 2: the real / imaginary part taken as a real column (the
// kx = 0 and kx = W/2 columns share packed column 0).
struct ColLoader {
    const float2* src;
    int h;
    int mode;
    ZF_DEV float2 operator()(int i) const {
        if (i >= h) return c_make(0.f, 0.f);
        if (mode == 0) return src[i];
        const float* f = reinterpret_cast<const float*>(src + i);
        return c_make(mode == 1 ? f[0] : f[1], 0.f);
    }
};

// Row input for the folded real FFT: z[m] = x[2m] + i x[2m+1], x zero past w.
struct RowLoader {
    const float* row;
    int w;
    ZF_DEV float2 operator()(int m) const {
        int i = 2 * m;
        float a = i < w ? __ldg(row + i) : 0.f;
        float b = i + 1 < w ? __ldg(row + i + 1) : 0.f;
        return c_make(a, b);
    }
};

// ---------------------------------------------------------------------------
// Kernel 1: forward real FFT of the template rows, folded into a W2-point
// complex FFT plus the split post-pass; output packed and scaled by `scale`.
// ---------------------------------------------------------------------------
template <int W2, int NZ>
__global__ void __launch_bounds__(RowCfg<W2>::THREADS)
    k_row_r2c(const float* __restrict__ tmpl, float2* __restrict__ ws,
              const float2* __restrict__ twW, int h, int w, int H, float scale) {
    using C = RowCfg<W2>;
    using F = Stockham<W2, C::T, false, false>;
    static_assert(F::S >= 2, "row FFT needs at least two stages");
    constexpr int RL = F::radix(F::S - 1), NBL = F::nbf(F::S - 1);

    const int tid = threadIdx.x;
    const int g = tid / C::T, t = tid % C::T;
    float2* smem = dyn_smem();
    float2* buf = smem + g * C::BUF;

    typename F::Twiddles tw;
    F::template load_twiddles<2 * W2>(tw, twW, t);

    for (int n0 = blockIdx.x * C::RPB; n0 < h; n0 += gridDim.x * C::RPB) {
        const int n = n0 + g;
        RowLoader ld{tmpl + (size_t)(n < h ? n : 0) * w, n < h ? w : 0};
        float2 v[F::MAXE];
        F::template run_loader<NZ>(v, ld, buf, tw, t);
        // Z in natural order into the buffer.
#pragma unroll
        for (int q = 0; q < F::bpt(F::S - 1); ++q) {
            int b = t + q * C::T;
            if (F::even(F::S - 1) || b < NBL) {
#pragma unroll
                for (int r = 0; r < RL; ++r) buf[spad(b + r * NBL)] = v[q * RL + r];
            }
        }
        __syncthreads();
        // Split pass: X[k] = E[k] + w^k O[k], X[W2-k] = conj(E[k] - w^k O[k]),
        // E = (Z[k] + conj Z[W2-k]) / 2, O = (Z[k] - conj Z[W2-k]) / 2i.
        // Items (k, row) with the row index fastest, so each store of a column
        // segment R[k][n0 .. n0+RPB) is contiguous.
        constexpr int NIT = (W2 / 2 + 1) * C::RPB;
        for (int it = tid; it < NIT; it += C::THREADS) {
            const int nl = it % C::RPB, k = it / C::RPB;
            const int nn = n0 + nl;
            if (nn >= h) continue;
            const float2* zb = smem + nl * C::BUF;
            const float2 A = zb[spad(k)];
            if (k == 0) {
                ws[nn] = c_make((A.x + A.y) * scale, (A.x - A.y) * scale);
                continue;
            }
            const float2 B = zb[spad(W2 - k)];
            const float2 E = c_make(0.5f * (A.x + B.x), 0.5f * (A.y - B.y));
            const float2 G = c_make(0.5f * (A.x - B.x), 0.5f * (A.y + B.y));  // (A - conj B)/2
            const float2 wk = __ldg(twW + k);
            const float2 Ow = c_mul(c_make(G.y, -G.x), wk);  // w^k * G / i
            ws[(size_t)k * H + nn] = c_scale(c_add(E, Ow), scale);
            if (2 * k != W2) ws[(size_t)(W2 - k) * H + nn] = c_scale(c_conj(c_sub(E, Ow)), scale);
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------------------
// Kernel 2: per packed column, forward FFT over H of the h non-zero rows,
// multiply by the conjugate (correlation) or plain (convolution) image
// spectrum column, inverse FFT, store the first store_rows rows in place.
// The block loops over columns; virtual column vc in [0, W2] is
//   vc = 0      : real column kx = 0   (real part of packed column 0)
//   vc = W2     : real column kx = W/2 (imaginary part of packed column 0)
//   otherwise   : complex column kx = vc.
// ---------------------------------------------------------------------------
template <int H, bool CONJ, int NZ>
__global__ void __launch_bounds__(ColCfg<H>::THREADS)
    k_col_fused(float2* __restrict__ ws, const float2* __restrict__ spec,
                const float2* __restrict__ twH, int h, int W2, int store_rows) {
    using C = ColCfg<H>;
    using F = Stockham<H, C::T, false, false>;
    using I = Stockham<H, C::T, true, true>;
    static_assert(F::S >= 2, "column FFT needs at least two stages");
    static_assert(F::radix(F::S - 1) == I::radix(0), "fused layouts must agree");
    constexpr int RL = F::radix(F::S - 1), NBL = F::nbf(F::S - 1);
    constexpr int RO = I::radix(I::S - 1), NBO = I::nbf(I::S - 1);

    const int tid = threadIdx.x;
    const int g = tid / C::T, t = tid % C::T;
    float2* buf = dyn_smem() + g * C::BUF;

    typename F::Twiddles twf;
    F::template load_twiddles<H>(twf, twH, t);
    constexpr bool kShare = plan_palindrome(H);
    typename I::Twiddles twi_own;
    if constexpr (!kShare) I::template load_twiddles<H>(twi_own, twH, t);

    for (int vc0 = blockIdx.x * C::FPB; vc0 <= W2; vc0 += gridDim.x * C::FPB) {
        const int vc = vc0 + g;
        const bool active = vc <= W2;
        const int mode = vc == 0 ? 1 : (vc == W2 ? 2 : 0);
        const size_t col = (size_t)(mode != 0 ? 0 : vc) * H;
        ColLoader ld{ws + col, active ? h : 0, mode};

        float2 v[F::MAXE];
        F::template run_loader<NZ>(v, ld, buf, twf, t);

        // Pointwise product with the image spectrum column (cuh:86-111).
        const float2* sp = spec + (size_t)(active ? vc : 0) * H;
#pragma unroll
        for (int q = 0; q < F::bpt(F::S - 1); ++q) {
            int b = t + q * C::T;
            if (F::even(F::S - 1) || b < NBL) {
#pragma unroll
                for (int r = 0; r < RL; ++r) {
                    float2 s = __ldg(sp + b + r * NBL);
                    float2 a = v[q * RL + r];
                    v[q * RL + r] = CONJ ? c_conj_mul(a, s) : c_mul(a, s);
                }
            }
        }

        if constexpr (kShare) {
            I::run_regs(v, buf, twf, t);
        } else {
            I::run_regs(v, buf, twi_own, t);
        }

        if (active) {
            float2* dst = ws + col;
            float* dstf = reinterpret_cast<float*>(dst);
#pragma unroll
            for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                int b = t + q * C::T;
                if (I::even(I::S - 1) || b < NBO) {
#pragma unroll
                    for (int r = 0; r < RO; ++r) {
                        int y = b + r * NBO;
                        if (y < store_rows) {
                            float2 o = v[q * RO + r];
                            if (mode == 0) {
                                dst[y] = o;
                            } else {
                                dstf[2 * y + (mode == 2 ? 1 : 0)] = o.x;
                            }
                        }
                    }
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Kernel 3: inverse real FFT of output rows, folded into a W2-point complex
// inverse FFT after the split pre-pass; crops to out_cols columns.
// ---------------------------------------------------------------------------
template <int W2>
__global__ void __launch_bounds__(RowCfg<W2>::THREADS)
    k_row_c2r(const float2* __restrict__ ws, float* __restrict__ out,
              const float2* __restrict__ twW, int H, int out_rows, int out_cols,
              int out_pitch) {
    using C = RowCfg<W2>;
    using I = Stockham<W2, C::T, true, false>;
    static_assert(I::S >= 2, "row FFT needs at least two stages");
    constexpr int RL = I::radix(I::S - 1), NBL = I::nbf(I::S - 1);

    const int tid = threadIdx.x;
    const int g = tid / C::T, t = tid % C::T;
    float2* smem = dyn_smem();
    float2* buf = smem + g * C::BUF;

    typename I::Twiddles tw;
    I::template load_twiddles<2 * W2>(tw, twW, t);

    const bool vec_ok = out_cols == 2 * W2 && (out_pitch % 2) == 0 &&
                        (reinterpret_cast<size_t>(out) % 8) == 0;

    for (int y0 = blockIdx.x * C::RPB; y0 < out_rows; y0 += gridDim.x * C::RPB) {
        // Split pre-pass: 2Z[k] = (X[k] + conj X[W2-k]) + i w^-k (X[k] - conj X[W2-k]).
        constexpr int NIT = (W2 / 2 + 1) * C::RPB;
        for (int it = tid; it < NIT; it += C::THREADS) {
            const int yl = it % C::RPB, k = it / C::RPB;
            const int y = y0 + yl;
            if (y >= out_rows) continue;
            float2* zb = smem + yl * C::BUF;
            const float2 A = ws[(size_t)k * H + y];
            if (k == 0) {  // packed (X[0], X[W2])
                zb[spad(0)] = c_make(A.x + A.y, A.x - A.y);
                continue;
            }
            const float2 B = ws[(size_t)(W2 - k) * H + y];
            const float2 E2 = c_make(A.x + B.x, A.y - B.y);  // A + conj B
            const float2 D = c_make(A.x - B.x, A.y + B.y);   // A - conj B
            const float2 P = c_mul_conj(D, __ldg(twW + k));   // w^-k D
            const float2 iP = c_mul_i(P);
            zb[spad(k)] = c_add(E2, iP);
            if (2 * k != W2) zb[spad(W2 - k)] = c_conj(c_sub(E2, iP));
        }
        __syncthreads();

        float2 v[I::MAXE];
        I::run_smem(v, buf, tw, t);

        const int y = y0 + g;
        if (y < out_rows) {
            float* orow = out + (size_t)y * out_pitch;
#pragma unroll
            for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                int b = t + q * C::T;
                if (I::even(I::S - 1) || b < NBL) {
#pragma unroll
                    for (int r = 0; r < RL; ++r) {
                        const int m = b + r * NBL;
                        const float2 z = v[q * RL + r];
                        if (vec_ok) {
                            reinterpret_cast<float2*>(orow)[m] = z;
                        } else {
                            if (2 * m < out_cols) orow[2 * m] = z.x;
                            if (2 * m + 1 < out_cols) orow[2 * m + 1] = z.y;
                        }
                    }
                }
            }
        }
    }
}

}  // namespace zf
