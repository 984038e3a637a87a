// The three kernels of the implicitly zero-padded real 2D FFT cross-correlation
// (zipFFT: src/cuda/real_conv_2d.cuh:6-117, I/O layer src/cuda/real_conv_2d_io.hpp).
//
// Per template, with image size H x W, template h x w and W2 = W/2:
//
//   k_row_r2c   rows n < h:  X_n = rfft_W(pad(t_n)) * 1/(H W)      (cuh:8-30)
//               stored column-major as R[kx][n], packed kx = 0..W2-1
//   k_col_fused columns kx:  Q[., kx] = IFFT_H( conj(FFT_H(pad_h(R[kx]))) . S[kx] )
//                                                                   (cuh:58-117)
//   k_row_c2r   rows y:      out[y] = irfft_W(Q[y, .]), cropped       (cuh:34-56)
//               epilogues: store the map (optionally folding its maximum into a
//               per-template peak), or fold it into running per-pixel max /
//               argmax (optionally sum / sum of squares) maps
//
// and, for the image spectrum the operator takes (conv_data), k_row_r2c over
// the image rows followed by
//
//   k_col_fwd   columns kx:  S[kx] = FFT_H(R[kx]), in place in conv_data
//
// Intermediate layout (complex64): Q is column-major, element (kx, y) at
// kx * H + y, packed kx in [0, W2), so one H x W2 slice holds a template's
// intermediate (the reference's workspace holds H x (W/2+1) per template,
// real_conv_2d_binding.cu:235-245).  Packed column 0 carries the two real
// columns kx = 0 (real part) and kx = W/2 (imaginary part).  R either sits in
// rows [0, h) of the same slice (pitch H; the column kernel then overwrites it
// in place, each column by the block that read it) or in a separate region
// with pitch round_up(h, 2) so that the row kernel can run several templates
// per launch.  With a workspace of several slices (batched groups), each
// kernel runs a group of templates per launch, template j in slice j with its
// R in rows [0, h) of that slice.
//
// Differences from the reference's data movement (io.hpp:134-195, which reads
// a row-major workspace down its columns at stride W/2+1):
//   * the column kernel streams whole contiguous columns: the image spectrum
//     column and the template column arrive by TMA bulk copies into shared
//     memory, double-buffered across the block's loop over columns;
//   * the inverse row kernel fetches 2-row x 256-column tiles of Q with 2D TMA
//     tensor loads (the transpose happens in the copy engine);
//   * the normalisations 1/H (io.hpp:278-282) and 1/W (io.hpp:302-306) are
//     folded into the template rows, so later kernels do no scaling.
#pragma once

#include "async_copy.cuh"
#include "fft_core.cuh"

namespace zf {

#if defined(__CUDACC__)
ZF_DEV float2* dyn_smem() {
    extern __shared__ __align__(128) float2 zf_dyn_smem_arr[];
    return zf_dyn_smem_arr;
}
#else
float2* dyn_smem();  // provided by the CPU test harness
#endif

// Threads per transform: 16 elements per thread in radix-16 stages.  For the
// sizes 15 * 2^k, n / 15 threads instead: the radix-5 and radix-3 stages then
// give every thread exactly 3 or 5 butterflies (15 elements) instead of a
// ragged 20, at the price of n / 240 idle threads in radix-16 stages.
constexpr int fft_threads(int n) { return n % 15 == 0 ? n / 15 : (n + 15) / 16; }
constexpr int round_up(int x, int m) { return (x + m - 1) / m * m; }
// Largest divisor of n that is at most cap.
constexpr int largest_divisor_upto(int n, int cap) {
    for (int d = cap; d > 1; --d)
        if (n % d == 0) return d;
    return 1;
}
constexpr int cmax(int a, int b) { return a > b ? a : b; }
// Padded exchange buffer length, = 4 (mod 16): buffers of consecutive rows then
// start 8 banks apart, so the split passes (which walk 4 rows in lockstep)
// are bank-conflict free.
constexpr int xbuf_len(int n) { return round_up(spad_size(n) - 4, 16) + 4; }

// True when the radix sequence of n reads the same backwards.  The column
// kernel's inverse runs the radices in reverse, so for such plans it can use
// the forward twiddles (conjugated by the inverse butterflies).
constexpr bool plan_palindrome(int n) {
    PlanInfo p = make_plan(n);
    for (int s = 0; s < p.S; ++s)
        if (p.R[s] != p.R[p.S - 1 - s]) return false;
    return true;
}

// ===========================================================================
// Kernel 1: forward real FFT of template rows (W2-point complex FFT of
// z[m] = x[2m] + i x[2m+1] plus the split post-pass), packed and scaled.
// The (template, row group) pairs of all ntemplates templates form one index
// space that a single wave of blocks strides through.
// ===========================================================================
template <int W2>
struct R2cCfg {
    static constexpr int T = fft_threads(W2);
    static constexpr int RPB = cmax(4, 256 / T);  // rows per block
    static constexpr int THREADS = RPB * T;
    static constexpr int XB = xbuf_len(W2);
    static constexpr int SMEM = RPB * XB * 8;
};

// Row input for the folded real FFT, zero past the template width.
struct RowLoader {
    const float* row;
    int w;
    ZF_DEV float2 operator()(int m) const {
        const int i = 2 * m;
        const float a = i < w ? __ldg(row + i) : 0.f;
        const float b = i + 1 < w ? __ldg(row + i + 1) : 0.f;
        return c_make(a, b);
    }
};

template <int W2, int NZ>
__global__ void __launch_bounds__(R2cCfg<W2>::THREADS)
    k_row_r2c(const float* __restrict__ tmpl, float2* __restrict__ R, const float2* __restrict__ twW,
              const float4* __restrict__ twt, int h, int w, int r_pitch, long long r_tstride,
              int ntemplates, float scale) {
    using C = R2cCfg<W2>;
    using F = Stockham<W2, C::T, false, false>;
    static_assert(F::S >= 2, "row FFT needs at least two stages");
    constexpr int RL = F::radix(F::S - 1), NBL = F::nbf(F::S - 1);

    const int tid = threadIdx.x;
    const int g = tid / C::T, t = tid % C::T;
    float2* smem = dyn_smem();
    float2* buf = smem + g * C::XB;

    pdl_launch_dependents();
    typename F::Twiddles tw;
    F::load_thread_twiddles(tw, twt, t);
    // R may still be read by the previous kernel of the stream.
    pdl_wait_prerequisites();

    // Row groups cover rows [0, round_up(h, 2)): the padding row of an odd h
    // is written as zeros by the split pass below.
    const int h_pad = (h + 1) & ~1;
    const int groups = (h_pad + C::RPB - 1) / C::RPB;
    const int units = groups * ntemplates;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int tj = u / groups, n0 = (u - tj * groups) * C::RPB;
        const float* tm = tmpl + (size_t)tj * h * w;
        float2* Rt = R + (size_t)tj * r_tstride;
        const int n = n0 + g;
        RowLoader ld{tm + (size_t)(n < h ? n : 0) * w, n < h ? w : 0};
        float2 v[F::MAXE];
        F::template run_loader<NZ>(v, ld, buf, tw, t);
        // Z in natural order into the buffer (all reads of the buffer by the
        // last stage completed at run_loader's final barrier).
#pragma unroll
        for (int q = 0; q < F::bpt(F::S - 1); ++q) {
            const int b = t + q * C::T;
            if (F::even(F::S - 1) || b < NBL) {
#pragma unroll
                for (int r = 0; r < RL; ++r) buf[spad(b + r * NBL)] = v[q * RL + r];
            }
        }
        __syncthreads();
        // Split pass: X[k] = E[k] + w^k O[k], X[W2-k] = conj(E[k] - w^k O[k]),
        // E = (Z[k] + conj Z[W2-k]) / 2, O = (Z[k] - conj Z[W2-k]) / 2i.
        // Items (k, row) run with the row fastest so each store of a column
        // segment R[k][n0 .. n0+RPB) is contiguous.
        constexpr int NIT = (W2 / 2 + 1) * C::RPB;
        for (int it = tid; it < NIT; it += C::THREADS) {
            const int nl = it % C::RPB, k = it / C::RPB;
            const int nn = n0 + nl;
            if (nn >= h) {
                // Row h of an odd-height template is the zero padding that
                // the column kernel's 16-byte copies also fetch.
                if (nn == h && (h & 1)) {
                    Rt[(size_t)k * r_pitch + nn] = c_make(0.f, 0.f);
                    if (k != 0 && 2 * k != W2) Rt[(size_t)(W2 - k) * r_pitch + nn] = c_make(0.f, 0.f);
                }
                continue;
            }
            const float2* zb = smem + nl * C::XB;
            const float2 A = zb[spad(k)];
            if (k == 0) {
                Rt[nn] = c_make((A.x + A.y) * scale, (A.x - A.y) * scale);
                continue;
            }
            const float2 B = zb[spad(W2 - k)];
            const float2 E = c_make(0.5f * (A.x + B.x), 0.5f * (A.y - B.y));
            const float2 G = c_make(0.5f * (A.x - B.x), 0.5f * (A.y + B.y));  // (A - conj B)/2
            const float2 wk = __ldg(twW + k);
            const float2 Ow = c_mul(c_make(G.y, -G.x), wk);  // w^k * G / i
            Rt[(size_t)k * r_pitch + nn] = c_scale(c_add(E, Ow), scale);
            if (2 * k != W2) Rt[(size_t)(W2 - k) * r_pitch + nn] = c_scale(c_conj(c_sub(E, Ow)), scale);
        }
        __syncthreads();
    }
}

// ===========================================================================
// Kernel 2: per packed column, forward FFT over H of the h non-zero rows,
// product with the conjugate (correlation) or plain (convolution) image
// spectrum column, inverse FFT, first store_rows rows stored.
//
// Virtual column vc in [0, W2]: vc = 0 is the real column kx = 0 (real part of
// packed column 0), vc = W2 the real column kx = W/2 (its imaginary part),
// otherwise the complex column kx = vc.  A block holds FPB columns; it loops
// over column groups, prefetching the next group's spectrum and template
// columns by TMA while it transforms the current one.
// ===========================================================================
template <int H, int NZ>
struct ColCfg {
    static constexpr int T = fft_threads(H);
    static constexpr int FPB = T >= 128 ? 1 : 128 / T;  // columns per block
    static constexpr int THREADS = FPB * T;
    static constexpr int MINB = cmax(1, 512 / THREADS);  // blocks per SM targeted
    static constexpr int XB = xbuf_len(H);
    static constexpr int SB = round_up(H, 16);                     // spectrum column
    static constexpr int NB0 = H / make_plan(H).R[0];
    static constexpr int RB = round_up(NZ > 0 ? NZ * NB0 : H, 16);  // template column
    static constexpr int FLOATS = FPB * (XB + 2 * SB + 2 * RB);
    static constexpr int SMEM = FLOATS * 8 + 2 * 8;  // + two mbarriers
};

template <int H, bool CONJ, int NZ>
__global__ void __launch_bounds__(ColCfg<H, NZ>::THREADS, ColCfg<H, NZ>::MINB)
    k_col_fused(float2* __restrict__ Q, const float2* __restrict__ R, int r_pitch,
                const float2* __restrict__ spec, const float4* __restrict__ twt,
                const float4* __restrict__ twt_rev, int h, int W2, int store_rows, int discard_r,
                int ntemplates, long long q_tstride, long long r_tstride,
                int* __restrict__ status) {
    using C = ColCfg<H, NZ>;
    using F = Stockham<H, C::T, false, false>;
    using I = Stockham<H, C::T, true, true>;
    static_assert(F::S >= 2, "column FFT needs at least two stages");
    static_assert(F::radix(F::S - 1) == I::radix(0), "fused layouts must agree");
    constexpr int RL = F::radix(F::S - 1), NBL = F::nbf(F::S - 1);
    constexpr int RO = I::radix(I::S - 1), NBO = I::nbf(I::S - 1);

    const int tid = threadIdx.x;
    const int g = tid / C::T, t = tid % C::T;
    float2* smem = dyn_smem();
    float2* xbuf = smem + g * C::XB;
    float2* sbase = smem + C::FPB * C::XB;            // [2][FPB][SB]
    float2* rbase = sbase + 2 * C::FPB * C::SB;       // [2][FPB][RB]
    uint64_t* mbar = reinterpret_cast<uint64_t*>(rbase + 2 * C::FPB * C::RB);

    // Template-column buffers are zero beyond h: the pruned start reads them
    // unconditionally.  TMA later overwrites only the first round_up(h, 2).
    for (int i = tid; i < 2 * C::FPB * C::RB; i += C::THREADS) rbase[i] = c_make(0.f, 0.f);
    __syncthreads();
    if (tid == 0) {  // after the zero fill: orders it before the first TMA write
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_init_fence();
    }
    __syncthreads();

    pdl_launch_dependents();
    typename F::Twiddles twf;
    F::load_thread_twiddles(twf, twt, t);
    constexpr bool kShare = plan_palindrome(H);
    typename I::Twiddles twi_own;
    if constexpr (!kShare) I::load_thread_twiddles(twi_own, twt_rev, t);
    const uint32_t r_bytes = (uint32_t)round_up(h, 2) * 8u;
    // Units (template, column group): ntemplates templates of W2 + 1 virtual
    // columns each, template j's Q and R at Q + j q_tstride, R + j r_tstride.
    // Column-major order: the templates of a column group are consecutive
    // units, so neighbouring blocks read the same spectrum columns at about
    // the same time and all but the first find them in L2.
    const int cgroups = (W2 + C::FPB) / C::FPB;
    const int units = cgroups * ntemplates;
    auto unit_cols = [&](int u, int& tj, int& vc0) {
        const int cg = u / ntemplates;
        tj = u - cg * ntemplates;
        vc0 = cg * C::FPB;
    };
    // L2 policy: template columns stream through (read once); the spectrum,
    // read once per template but by every template, keeps the normal policy
    // (some of it then survives in L2 for the next template: measured faster
    // than evict-first or evict-last); the intermediate Q is kept resident
    // for the row kernel that reads it next (with a group of templates per
    // launch as well: evict-first Q lines measured 1.7x slower there).
    const uint64_t pol_stream = l2_evict_first();
    const uint64_t pol_spec = l2_evict_normal();
    const uint64_t pol_keep = l2_evict_last();

    // Thread 0 fetches the spectrum and template columns of unit u into
    // buffer b: the spectrum part (which no kernel writes) and the template
    // part (written by the row kernel before this one) separately, both
    // completing on the buffer's barrier.
    auto issue_spec = [&](int b, int u) {
        int tj, vc0;
        unit_cols(u, tj, vc0);
        uint32_t bytes = 0;
        for (int j = 0; j < C::FPB; ++j)
            if (vc0 + j <= W2) bytes += H * 8u + r_bytes;
        mbar_arrive_expect_tx(&mbar[b], bytes);
        for (int j = 0; j < C::FPB; ++j) {
            const int vc = vc0 + j;
            if (vc > W2) break;
            tma_load_1d(sbase + (b * C::FPB + j) * C::SB, spec + (size_t)vc * H, H * 8u, &mbar[b],
                        pol_spec);
        }
    };
    auto issue_r = [&](int b, int u) {
        int tj, vc0;
        unit_cols(u, tj, vc0);
        const float2* Rj = R + tj * r_tstride;
        for (int j = 0; j < C::FPB; ++j) {
            const int vc = vc0 + j;
            if (vc > W2) break;
            const int rc = vc == W2 ? 0 : vc;
            tma_load_1d(rbase + (b * C::FPB + j) * C::RB, Rj + (size_t)rc * r_pitch, r_bytes,
                        &mbar[b], pol_stream);
        }
    };
    auto issue = [&](int b, int u) {
        issue_spec(b, u);
        issue_r(b, u);
    };

    // The first unit's spectrum columns do not depend on the previous kernel:
    // their copy overlaps its tail.  R comes from the previous kernel; Q may
    // still be read by the one before.
    if (tid == 0 && (int)blockIdx.x < units) issue_spec(0, blockIdx.x);
    pdl_wait_prerequisites();

    // Double buffering: thread 0 refills the other pair of buffers with the
    // next group once the block is past this group's barrier (their last
    // readers are behind it) and the previous column's bulk store, staged in
    // the other spectrum buffer, has read it; the block never waits for that
    // store.  (Refilling before the wait, or filling both buffers up front,
    // measured slower.)
    int u = blockIdx.x;
    if (tid == 0 && u < units) issue_r(0, u);
    for (int it = 0; u < units; ++it, u += gridDim.x) {
        const int b = it & 1;
        const uint32_t parity = (it >> 1) & 1;
        int tj, vc0;
        unit_cols(u, tj, vc0);
        float2* Qj = Q + tj * q_tstride;
        const float2* Rj = R + tj * r_tstride;
        const bool more = u + (int)gridDim.x < units;
        const bool ok = mbar_wait_bounded(&mbar[b], parity);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                atomicExch(status, kStatusTimeout);
                // The late copy may still land (the next one was not issued):
                // wait for it, bounded, before the block's memory is released.
                mbar_wait_bounded(&mbar[b], parity);
                bulk_wait_all();
            }
            return;
        }
        if (tid == 0 && more) {
            bulk_wait_read();
            issue(b ^ 1, u + gridDim.x);
        }

        const int vc = vc0 + g;
        const bool active = vc <= W2;
        const int mode = vc == 0 ? 1 : (vc == W2 ? 2 : 0);
        const float2* rcol = rbase + (b * C::FPB + g) * C::RB;
        const float2* scol = sbase + (b * C::FPB + g) * C::SB;
        // A template column outside Q (the chunked layout) has no other reader
        // once copied: drop its whole 128-byte lines from L2 without write-back.
        // Packed column 0 is read by two column kinds and is kept.
        if (discard_r && active && mode == 0) {
            const char* c0 = reinterpret_cast<const char*>(Rj + (size_t)vc * r_pitch);
            const size_t lo = (reinterpret_cast<size_t>(c0) + 127) & ~size_t(127);
            const size_t hi = (reinterpret_cast<size_t>(c0) + r_bytes) & ~size_t(127);
            for (size_t a = lo + (size_t)t * 128; a < hi; a += (size_t)C::T * 128)
                l2_discard_line(reinterpret_cast<const void*>(a));
        }

        // The template buffer is zero past h (zero fill beyond the copied
        // length; the row kernel writes the padding row of an odd h), so the
        // loader reads it unconditionally.
        float2 v[F::MAXE];
        if constexpr (C::FPB == 1) {
            // The column kind is uniform across the block: branching on it
            // keeps the block barriers inside the transform convergent.
            if (mode == 0) {
                auto ld = [&](int i) { return rcol[i]; };
                F::template run_loader<NZ>(v, ld, xbuf, twf, t);
            } else {
                const float* rf = reinterpret_cast<const float*>(rcol) + (mode == 2 ? 1 : 0);
                auto ld = [&](int i) { return c_make(rf[2 * i], 0.f); };
                F::template run_loader<NZ>(v, ld, xbuf, twf, t);
            }
        } else {
            // Groups of one block may hold different column kinds: one loader
            // with per-element selects, so every thread reaches the block
            // barriers inside the transform through the same instructions.
            const bool take_im = mode == 2, keep_im = mode == 0;
            auto ld = [&](int i) {
                const float2 x = rcol[i];
                return c_make(take_im ? x.y : x.x, keep_im ? x.y : 0.f);
            };
            F::template run_loader<NZ>(v, ld, xbuf, twf, t);
        }

        // Pointwise product with the image spectrum column (cuh:86-111).
#pragma unroll
        for (int q = 0; q < F::bpt(F::S - 1); ++q) {
            const int bb = t + q * C::T;
            if (F::even(F::S - 1) || bb < NBL) {
                const float2* sp = scol + bb;
#pragma unroll
                for (int r = 0; r < RL; ++r) {
                    const float2 s = sp[r * NBL];
                    const float2 a = v[q * RL + r];
                    v[q * RL + r] = CONJ ? c_conj_mul(a, s) : c_mul(a, s);
                }
            }
        }

        // No barrier after the inverse's last exchange: the next write of the
        // exchange buffer is the next group's transform, behind the loop-top
        // barrier (the staged column goes to the spectrum buffer).
        if constexpr (kShare) {
            I::template run_regs<false>(v, xbuf, twf, t);
        } else {
            I::template run_regs<false>(v, xbuf, twi_own, t);
        }

        if constexpr (C::FPB == 1) {
            if (mode == 0) {  // block-uniform (one column per block)
                // Stage the column in this group's spectrum buffer (read only
                // by the product, before the inverse transform's barriers) and
                // store it with one bulk copy; the exchange buffer is then free
                // for the next column at once.
                float2* stage = sbase + b * C::FPB * C::SB;
#pragma unroll
                for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                    const int bb = t + q * C::T;
                    if (I::even(I::S - 1) || bb < NBO) {
#pragma unroll
                        for (int r = 0; r < RO; ++r) stage[bb + r * NBO] = v[q * RO + r];
                    }
                }
                fence_proxy_async();
                __syncthreads();
                if (tid == 0) {
                    const int rows = store_rows >= H ? H : ((store_rows + 1) & ~1);
                    tma_store_1d(Qj + (size_t)vc * H, stage, (uint32_t)rows * 8u, pol_keep);
                    bulk_commit();
                }
                continue;
            }
        }
        if (active) {
            const bool full = store_rows >= H;
            if (mode == 0) {
                float2* dst = Qj + (size_t)vc * H;
#pragma unroll
                for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                    const int bb = t + q * C::T;
                    if (I::even(I::S - 1) || bb < NBO) {
#pragma unroll
                        for (int r = 0; r < RO; ++r) {
                            const int y = bb + r * NBO;
                            if (full || y < store_rows) st_hint(dst + y, v[q * RO + r], pol_keep);
                        }
                    }
                }
            } else {
                float* dstf = reinterpret_cast<float*>(Qj) + (mode == 2 ? 1 : 0);
#pragma unroll
                for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                    const int bb = t + q * C::T;
                    if (I::even(I::S - 1) || bb < NBO) {
#pragma unroll
                        for (int r = 0; r < RO; ++r) {
                            const int y = bb + r * NBO;
                            if (full || y < store_rows) st_hint(dstf + 2 * y, v[q * RO + r].x, pol_keep);
                        }
                    }
                }
            }
        }
    }
    if (tid == 0) bulk_wait_all();
}

// ===========================================================================
// Image spectrum, column pass (the operator's callers compute the spectrum as
// rfftn(image).transpose(-2, -1): zipFFT README.md:224-228, test:89-90).  The
// row kernel has written the image rows' real FFTs column-major into the
// (W/2+1, H) output itself -- packed column kx in [0, W2), element (kx, y) at
// kx * H + y -- and this kernel replaces each column by its forward H-point
// FFT, in place: a column is read (by TMA) and rewritten only by the block
// that owns it.  Packed column 0 holds P = X[., 0] + i X[., W/2] of two real
// columns, whose spectra separate as
//   S[0][k]    = (P^[k] + conj P^[-k]) / 2,
//   S[W/2][k]  = (P^[k] - conj P^[-k]) / 2i,
// the second into row W2 of the output, which no block reads.
// ===========================================================================
template <int H>
struct ColFwdCfg {
    static constexpr int T = fft_threads(H);
    static constexpr int FPB = T >= 128 ? 1 : 128 / T;  // columns per block
    static constexpr int THREADS = FPB * T;
    static constexpr int MINB = cmax(1, 512 / THREADS);
    static constexpr int XB = xbuf_len(H);
    static constexpr int CB = round_up(H, 16);  // one input column
    static constexpr int FLOATS = FPB * (XB + 2 * CB);
    static constexpr int SMEM = FLOATS * 8 + 2 * 8;  // + two mbarriers
};

template <int H>
__global__ void __launch_bounds__(ColFwdCfg<H>::THREADS, ColFwdCfg<H>::MINB)
    k_col_fwd(float2* __restrict__ spec, const float4* __restrict__ twt, int W2,
              int* __restrict__ status) {
    using C = ColFwdCfg<H>;
    using F = Stockham<H, C::T, false, false>;
    static_assert(F::S >= 2, "column FFT needs at least two stages");
    constexpr int RL = F::radix(F::S - 1), NBL = F::nbf(F::S - 1);

    const int tid = threadIdx.x;
    const int g = tid / C::T, t = tid % C::T;
    float2* smem = dyn_smem();
    float2* xbuf = smem + g * C::XB;
    float2* cbase = smem + C::FPB * C::XB;  // [2][FPB][CB]
    uint64_t* mbar = reinterpret_cast<uint64_t*>(cbase + 2 * C::FPB * C::CB);

    // Groups past the last column transform stale buffers: start them at zero.
    for (int i = tid; i < 2 * C::FPB * C::CB; i += C::THREADS) cbase[i] = c_make(0.f, 0.f);
    __syncthreads();
    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_init_fence();
    }
    __syncthreads();

    pdl_launch_dependents();
    typename F::Twiddles tw;
    F::load_thread_twiddles(tw, twt, t);
    // The row pass over the image wrote the columns.
    pdl_wait_prerequisites();

    const int stride = gridDim.x * C::FPB;
    const uint64_t pol_stream = l2_evict_first();
    auto issue = [&](int b, int c0) {
        uint32_t bytes = 0;
        for (int j = 0; j < C::FPB; ++j)
            if (c0 + j < W2) bytes += H * 8u;
        mbar_arrive_expect_tx(&mbar[b], bytes);
        for (int j = 0; j < C::FPB && c0 + j < W2; ++j)
            tma_load_1d(cbase + (b * C::FPB + j) * C::CB, spec + (size_t)(c0 + j) * H, H * 8u,
                        &mbar[b], pol_stream);
    };

    int c0 = blockIdx.x * C::FPB;
    if (tid == 0 && c0 < W2) issue(0, c0);
    for (int it = 0; c0 < W2; ++it, c0 += stride) {
        const int b = it & 1;
        const uint32_t parity = (it >> 1) & 1;
        // The other buffer was last read before this iteration's barrier.
        const bool more = c0 + stride < W2;
        if (tid == 0 && more) issue(b ^ 1, c0 + stride);
        const bool ok = mbar_wait_bounded(&mbar[b], parity);
        // Also orders the previous iteration's reads of xbuf before this
        // iteration's transform writes it.
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                atomicExch(status, kStatusTimeout);
                if (more) mbar_wait_bounded(&mbar[b ^ 1], ((it + 1) >> 1) & 1);
            }
            return;
        }

        const int kx = c0 + g;
        const float2* col = cbase + (b * C::FPB + g) * C::CB;
        float2 v[F::MAXE];
        auto ld = [&](int i) { return col[i]; };
        // With one column per block the column index is block-uniform: only
        // the block holding packed column 0 writes the exchange buffer after
        // the transform, so only it needs the barrier after the last
        // exchange (every block's next write of the buffer is behind the
        // loop-top barrier).  Blocks of several columns keep the barrier.
        constexpr bool kUniform = C::FPB == 1;
        F::template run_loader<0, !kUniform>(v, ld, xbuf, tw, t);
        if constexpr (kUniform) {
            if (kx == 0) __syncthreads();
        }

        // Frequency k = bb + r * NBL sits in v[q * RL + r].
        if (kx == 0) {
#pragma unroll
            for (int q = 0; q < F::bpt(F::S - 1); ++q) {
                const int bb = t + q * C::T;
                if (F::even(F::S - 1) || bb < NBL) {
#pragma unroll
                    for (int r = 0; r < RL; ++r) xbuf[bb + r * NBL] = v[q * RL + r];
                }
            }
        } else if (kx < W2) {
            float2* dst = spec + (size_t)kx * H;
#pragma unroll
            for (int q = 0; q < F::bpt(F::S - 1); ++q) {
                const int bb = t + q * C::T;
                if (F::even(F::S - 1) || bb < NBL) {
#pragma unroll
                    for (int r = 0; r < RL; ++r) dst[bb + r * NBL] = v[q * RL + r];
                }
            }
        }
        if (!kUniform || kx == 0) __syncthreads();  // block-uniform
        if (kx == 0) {  // split the packed column (its reads ended at the barrier above)
            float2* s0 = spec;
            float2* sn = spec + (size_t)W2 * H;
            for (int k = t; k < H; k += C::T) {
                const float2 p = xbuf[k];
                const float2 m = xbuf[k == 0 ? 0 : H - k];
                s0[k] = c_make(0.5f * (p.x + m.x), 0.5f * (p.y - m.y));
                sn[k] = c_make(0.5f * (p.y + m.y), 0.5f * (m.x - p.x));
            }
        }
    }
}

// ===========================================================================
// Kernel 3: inverse real FFT of output rows: the split pre-pass
//   2Z[k] = (X[k] + conj X[W2-k]) + i w^-k (X[k] - conj X[W2-k])
// is fused into the reads of the first stage; a W2-point complex inverse FFT
// follows; z[m] = (out[2m], out[2m+1]).  Each block loops over groups of RPB
// rows; a group's Q tile (all W2 columns x RPB rows) arrives by 2D TMA loads,
// double-buffered.
// ===========================================================================
// L2 prefetch of the whole 16-byte chunks inside the n floats at p.
ZF_DEV void prefetch_row(const float* p, int n) {
    const size_t a = (reinterpret_cast<size_t>(p) + 15) & ~size_t(15);
    const size_t e = reinterpret_cast<size_t>(p + n) & ~size_t(15);
    if (e > a) l2_prefetch_bulk(reinterpret_cast<const void*>(a), (uint32_t)(e - a));
}

// Largest divisor of n not above 256 (the TMA box limit).
constexpr int tma_box(int n) {
    for (int d = 256; d >= 1; --d)
        if (n % d == 0) return d;
    return 1;
}

template <int W2>
struct C2rCfg {
    static constexpr int T = fft_threads(W2);
    // rows per block (even: TMA x alignment); two blocks of 256 threads per SM
    // at W2 = 2048.
    static constexpr int RPB = cmax(2, (128 / T) & ~1);
    static constexpr int THREADS = RPB * T;
    static constexpr int MINB = cmax(1, 512 / THREADS);
    // Rows are interleaved across lanes (row = tid % RPB): the tile reads of
    // the pre-pass are then contiguous across a warp.  With two rows, row
    // buffers 16 banks apart keep the stage exchanges conflict free.
    static constexpr int XB = RPB == 2 ? round_up(spad_size(W2) - 8, 16) + 8 : xbuf_len(W2);
    static constexpr int BOXK = tma_box(W2);
    static constexpr int QB = round_up(W2 * RPB, 16);  // one Q tile
    static constexpr int FLOATS = 2 * QB + RPB * XB;
    // + two mbarriers + 32 floats for the block's peak reduction
    static constexpr int SMEM = FLOATS * 8 + 2 * 8 + 32 * 4;
};

// Epilogues of the inverse row pass.
constexpr int kStoreMap = 0;  // write the correlation map
constexpr int kRunningMax = 1;  // fold it into a running per-pixel max / argmax
constexpr int kRunningStats = 2;  // ... and into per-pixel sum and sum of squares
constexpr int kStorePeak = 3;  // write the map and fold its maximum into *peak
constexpr int kRunningSumSq = 4;  // as kRunningStats without the sum (sum of squares only)


// Maximum that returns NaN when either argument is NaN (as torch.amax does),
// unlike fmaxf.  fold_block_peak gives every NaN (of either sign: arithmetic
// on a NaN input may set its sign bit) the largest key, so it survives
// atomicMax and converts back to a NaN peak.
#if defined(__CUDA_ARCH__)
ZF_DEV float fmax_nan(float a, float b) {
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
    return r;
}
#else
inline float fmax_nan(float a, float b) { return (a != a || b != b) ? a + b : (a > b ? a : b); }
#endif

// kStorePeak: each thread keeps its largest stored value over the row groups
// of one template; the block folds them into that template's key (one atomic
// per block) when it moves on to another template or ends.  An atomic per
// warp and group put ~16k atomics on one address per 4096-row template, which
// serialised in L2; one per warp still slowed launches of many templates,
// whose keys share one L2 line.  Every thread of the block must call this
// (block-uniform); red: 32 floats of shared memory.  A block that gives up on
// a bounded wait folds what it has before it returns; the peaks of such a call
// are incomplete (the device status word reports it).
ZF_DEV void fold_block_peak(float v, unsigned* key, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmax_nan(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    if (lane == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        float x = lane < (int)(blockDim.x >> 5) ? red[lane] : -INFINITY;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) x = fmax_nan(x, __shfl_xor_sync(0xffffffffu, x, o));
        if (lane == 0) atomicMax(key, x != x ? 0xFFFFFFFFu : ordered_key(x));
    }
    __syncthreads();  // red is free again
}

// MODE kStoreMap: out[y][x] = correlation.  MODE kRunningMax: out is the
// running maximum map and arg the template-index map (same pitch); where the
// correlation is strictly greater than the stored maximum (or everywhere when
// reset & kResetMax), the maximum becomes the correlation and the index
// `tindex`.  Templates folded in increasing index order therefore keep the
// lowest index on ties.  MODE kRunningStats: as kRunningMax, and the
// correlation and its square are also added to the maps sum and sumsq (same
// pitch; reset & (kResetMax | kResetSums) overwrites them instead, so that a
// caller can start float32 partial sums per batch and accumulate the batches
// at higher precision while the maximum keeps running).  MODE kRunningSumSq:
// as kRunningStats without the sum map (sum unused).
//
// Several templates per launch: in the map modes the units (template, row
// group) are strided over the grid.  In the running-map modes each block owns
// whole row groups and folds the launch's templates into a group one after
// another, template j with index tindex + j (reset applies to j = 0 only):
// every pixel's updates then come from one block in template order (ties keep
// the lowest index), and the group's map rows stay hot in L2 across the
// templates instead of making a DRAM round trip per template.
template <int W2, int MODE>
__global__ void __launch_bounds__(C2rCfg<W2>::THREADS, C2rCfg<W2>::MINB)
    k_row_c2r(const __grid_constant__ CUtensorMap qmap, float* __restrict__ out,
              int* __restrict__ arg, float* __restrict__ sum, float* __restrict__ sumsq,
              unsigned* __restrict__ peak, const float2* __restrict__ twW,
              const float4* __restrict__ twt, int out_rows, int out_cols, int out_pitch,
              int tindex, int reset, int ntemplates, long long out_tstride,
              int* __restrict__ status) {
    using C = C2rCfg<W2>;
    using I = Stockham<W2, C::T, true, false>;
    static_assert(I::S >= 2, "row FFT needs at least two stages");
    constexpr int R0 = I::radix(0), NB0 = I::nbf(0);
    constexpr int RL = I::radix(I::S - 1), NBL = I::nbf(I::S - 1);
    static_assert((C::RPB * 8) % 16 == 0, "TMA inner box must be a multiple of 16 bytes");

    const int tid = threadIdx.x;
    const int g = tid % C::RPB, t = tid / C::RPB;
    float2* smem = dyn_smem();
    float2* qbase = smem;                       // [2][W2][RPB]
    float2* xbuf = smem + 2 * C::QB + g * C::XB;
    uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + C::FLOATS);
    float* red = reinterpret_cast<float*>(mbar + 2);  // kStorePeak's block reduction

    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_init_fence();
    }
    __syncthreads();

    pdl_launch_dependents();
    typename I::Twiddles tw;
    I::load_thread_twiddles(tw, twt, t);
    // Pre-pass twiddles w_W^-k for k = bb + r NB0: w^-bb (per butterfly, from
    // the table) times w_W^-(r NB0) = w_{2 R0}^-r (compile-time roots).
    float2 wpre[I::bpt(0)];
#pragma unroll
    for (int q = 0; q < I::bpt(0); ++q) {
        const int bb = t + q * C::T;
        wpre[q] = (I::even(0) || bb < NB0) ? c_conj(__ldg(twW + bb)) : c_make(1.f, 0.f);
    }
    // Q comes from the previous kernel.
    pdl_wait_prerequisites();

    // Units (template, row group): template j's Q is columns [j W2, (j+1) W2)
    // of the tile map, its map out + j out_tstride and its peak peak[j].
    // This block's k-th unit: see the kernel's comment for the two orders.
    constexpr bool kRunning = MODE == kRunningMax || MODE == kRunningStats || MODE == kRunningSumSq;
    const int ngroups = (out_rows + C::RPB - 1) / C::RPB;
    const int units = ngroups * ntemplates;
    auto unit_of = [&](int k, int& tj, int& grp) -> bool {
        if constexpr (kRunning) {
            tj = k % ntemplates;
            grp = (int)blockIdx.x + (k / ntemplates) * (int)gridDim.x;
            return grp < ngroups;
        } else {
            const int uu = (int)blockIdx.x + k * (int)gridDim.x;
            tj = uu / ngroups;
            grp = uu - tj * ngroups;
            return uu < units;
        }
    };

    // L2 policy: Q lines stay resident (the next template's column pass
    // overwrites them there without a DRAM round trip); output rows stream out.
    const uint64_t pol_keep = l2_evict_last();
    const uint64_t pol_stream = l2_evict_first();
    auto issue = [&](int b, int tj, int grp) {
        mbar_arrive_expect_tx(&mbar[b], (uint32_t)(W2 * C::RPB * 8));
        for (int k0 = 0; k0 < W2; k0 += C::BOXK)
            tma_load_2d(qbase + b * C::QB + k0 * C::RPB, &qmap, grp * C::RPB, tj * W2 + k0,
                        &mbar[b], pol_keep);
    };

    // Output rows leave through per-thread stores: staging them for bulk
    // stores needs one more block barrier per group, which cost more than the
    // store-queue stalls it removed.
    // Running-map modes: L2 prefetch of the rows of the maps that row group
    // grp's epilogue reads (once per group: its templates follow one another).
    auto prefetch_maps = [&](int grp) {
        const int g0 = grp * C::RPB;
        for (int r = 0; r < C::RPB; ++r) {
            const int yy = g0 + r;
            if (yy >= out_rows) break;
            prefetch_row(out + (size_t)yy * out_pitch, out_cols);
            if constexpr (MODE == kRunningStats) prefetch_row(sum + (size_t)yy * out_pitch, out_cols);
            if constexpr (MODE == kRunningStats || MODE == kRunningSumSq)
                prefetch_row(sumsq + (size_t)yy * out_pitch, out_cols);
        }
    };

    int tj = 0, grp = 0;
    bool have = unit_of(0, tj, grp);
    if (tid == 0 && have) issue(0, tj, grp);
    if constexpr (kRunning) {
        if (tid == 0 && have) prefetch_maps(grp);
    }
    float pk_run = -INFINITY;  // kStorePeak: this thread's largest value of template pk_t so far
    int pk_t = -1;
    for (int it = 0; have; ++it) {
        int next_tj = 0, next_grp = 0;
        const bool more = unit_of(it + 1, next_tj, next_grp);
        float* outj = out + tj * out_tstride;
        // Running modes: template j of this launch has index tindex + j, and
        // only the launch's first template resets the maps.
        [[maybe_unused]] const int reset_j = tj == 0 ? reset : 0;
        [[maybe_unused]] const int index_j = tindex + tj;
        if constexpr (MODE == kStorePeak) {
            if (pk_t >= 0 && pk_t != tj) {  // block-uniform
                fold_block_peak(pk_run, peak + pk_t, red);
                pk_run = -INFINITY;
            }
            pk_t = tj;
        }
        const int b = it & 1;
        const uint32_t parity = (it >> 1) & 1;
        if (tid == 0 && more) issue(b ^ 1, next_tj, next_grp);
        if constexpr (kRunning) {
            // The maps the NEXT group's epilogue reads: into L2 a whole
            // iteration ahead (whole 16-byte chunks inside each row only).
            // The first group's were requested before the loop.
            if (tid == 0 && more && next_grp != grp) prefetch_maps(next_grp);
        }
        const bool ok = mbar_wait_bounded(&mbar[b], parity);
        if (__syncthreads_or(!ok)) {  // block-uniform: every lane folds its warp
            if constexpr (MODE == kStorePeak) {
                if (pk_t >= 0) fold_block_peak(pk_run, peak + pk_t, red);
            }
            if (tid == 0) {
                atomicExch(status, kStatusTimeout);
                if (more) mbar_wait_bounded(&mbar[b ^ 1], ((it + 1) >> 1) & 1);
            }
            return;
        }

        // Stage 0 reads with the split pre-pass fused in: element k of row g.
        const float2* qt = qbase + b * C::QB + g;
        float2 v[I::MAXE];
#pragma unroll
        for (int q = 0; q < I::bpt(0); ++q) {
            const int bb = t + q * C::T;
            if (I::even(0) || bb < NB0) {
                const float2 wb = wpre[q];
                static_for<R0>([&](auto rc) {
                    constexpr int r = decltype(rc)::value;
                    const int k = bb + r * NB0;
                    const float2 A = qt[k * C::RPB];
                    const float2 B = qt[((W2 - k) % W2) * C::RPB];
                    const float2 E2 = px_fma(B, c_make(1.f, -1.f), A);  // A + conj B
                    const float2 D = px_fma(B, c_make(-1.f, 1.f), A);   // A - conj B
                    // z = E2 + i P with P = w^-k D = (w^-bb D) w_{2 R0}^-r; the
                    // constant root is folded into the sum when it is +-i.
                    const float2 Pb = c_mul(D, wb);
                    float2 z;
                    if constexpr (is_quarter_turn<2 * R0 - r, 2 * R0, false>()) {
                        // i (+-i) Pb = -+Pb
                        z = quarter_turn_inv<2 * R0 - r, 2 * R0, false>() ? c_sub(E2, Pb)
                                                                          : c_add(E2, Pb);
                    } else {
                        const float2 P = c_mul_w<2 * R0 - r, 2 * R0, false>(Pb);
                        z = px_fma(c_swap(P), c_make(-1.f, 1.f), E2);  // E2 + i P
                    }
                    if (r == 0 && bb == 0) z = c_make(A.x + A.y, A.x - A.y);  // packed (X0, X_W2)
                    v[q * R0 + r] = z;
                });
            }
        }
        // No barrier after the last exchange: the epilogue uses registers and
        // global memory only, and the next group's first write of the
        // exchange buffer is behind the loop-top barrier.
        I::template run_regs<false>(v, xbuf, tw, t);

        const int y = grp * C::RPB + g;
        float pk = -INFINITY;  // kStorePeak: this thread's largest stored value
        if (y < out_rows) {
            float* orow = outj + (size_t)y * out_pitch;
            // Element m holds outputs 2m, 2m+1: one 8-byte access where the
            // row is 8-byte aligned and both lie inside the crop.  With an odd
            // pitch every other row qualifies.
            auto aligned8 = [](const void* p) { return (reinterpret_cast<size_t>(p) & 7) == 0; };
            if constexpr (MODE == kStoreMap || MODE == kStorePeak) {
                const bool rv = aligned8(orow);
                // Full aligned rows (the common case) take a branch-free copy
                // of the loop; cropped or misaligned rows test each pair.
                auto emit = [&](auto full_row) {
                    constexpr bool FULL = decltype(full_row)::value;
#pragma unroll
                    for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                        const int bb = t + q * C::T;
                        if (I::even(I::S - 1) || bb < NBL) {
#pragma unroll
                            for (int r = 0; r < RL; ++r) {
                                const int m = bb + r * NBL;
                                const float2 z = v[q * RL + r];
                                if (FULL || (rv && 2 * m + 1 < out_cols)) {
                                    st_hint(reinterpret_cast<float2*>(orow) + m, z, pol_stream);
                                    if constexpr (MODE == kStorePeak) pk = fmax_nan(pk, fmax_nan(z.x, z.y));
                                } else {
                                    if (2 * m < out_cols) {
                                        st_hint(orow + 2 * m, z.x, pol_stream);
                                        if constexpr (MODE == kStorePeak) pk = fmax_nan(pk, z.x);
                                    }
                                    if (2 * m + 1 < out_cols) {
                                        st_hint(orow + 2 * m + 1, z.y, pol_stream);
                                        if constexpr (MODE == kStorePeak) pk = fmax_nan(pk, z.y);
                                    }
                                }
                            }
                        }
                    }
                };
                if (rv && out_cols == 2 * W2)
                    emit(std::true_type{});
                else
                    emit(std::false_type{});
            } else {
                int* arow = arg + (size_t)y * out_pitch;
                const bool rv = aligned8(orow) && aligned8(arow);
                // A chunk of a butterfly's outputs at a time, loads of the
                // stored values first, then the updates (all of them at once
                // held too many registers).
                constexpr int MCH = largest_divisor_upto(RL, 8);
#pragma unroll
                for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                    const int bb = t + q * C::T;
                    if (!(I::even(I::S - 1) || bb < NBL)) continue;
#pragma unroll
                    for (int r0 = 0; r0 < RL; r0 += MCH) {
                        float2 cur[MCH];
#pragma unroll
                        for (int i = 0; i < MCH; ++i) {
                            const int m = bb + (r0 + i) * NBL;
                            float2 c = c_make(-INFINITY, -INFINITY);
                            if (!(reset_j & kResetMax)) {
                                if (rv && 2 * m + 1 < out_cols) {
                                    c = reinterpret_cast<const float2*>(orow)[m];
                                } else {
                                    if (2 * m < out_cols) c.x = orow[2 * m];
                                    if (2 * m + 1 < out_cols) c.y = orow[2 * m + 1];
                                }
                            }
                            cur[i] = c;
                        }
#pragma unroll
                        for (int i = 0; i < MCH; ++i) {
                            const int m = bb + (r0 + i) * NBL;
                            const float2 z = v[q * RL + r0 + i];
                            const float2 c = cur[i];
                            const bool rmax = (reset_j & kResetMax) != 0;
                            const bool u0 = rmax || z.x > c.x, u1 = rmax || z.y > c.y;
                            if (rv && 2 * m + 1 < out_cols) {
                                if (u0 && u1) {
                                    reinterpret_cast<float2*>(orow)[m] = z;
                                    reinterpret_cast<int2*>(arow)[m] = make_int2(index_j, index_j);
                                } else if (u0) {
                                    orow[2 * m] = z.x;
                                    arow[2 * m] = index_j;
                                } else if (u1) {
                                    orow[2 * m + 1] = z.y;
                                    arow[2 * m + 1] = index_j;
                                }
                            } else {
                                if (u0 && 2 * m < out_cols) {
                                    orow[2 * m] = z.x;
                                    arow[2 * m] = index_j;
                                }
                                if (u1 && 2 * m + 1 < out_cols) {
                                    orow[2 * m + 1] = z.y;
                                    arow[2 * m + 1] = index_j;
                                }
                            }
                        }
                    }
                }
                if constexpr (MODE == kRunningStats || MODE == kRunningSumSq) {
                    // Per-pixel sum and sum of squares (float accumulation);
                    // a chunk of a butterfly's outputs at a time, loads first.
                    // kRunningSumSq: the sum of squares alone (a caller can
                    // get the sum of a batch's maps as the map of the batch's
                    // summed template, correlation being linear).
                    constexpr bool with_sum = MODE == kRunningStats;
                    float* srow = with_sum ? sum + (size_t)y * out_pitch : nullptr;
                    float* qrow = sumsq + (size_t)y * out_pitch;
                    const bool rvs = (!with_sum || aligned8(srow)) && aligned8(qrow);
                    const bool fresh = (reset_j & (kResetMax | kResetSums)) != 0;
                    constexpr int SCH = largest_divisor_upto(RL, 4);
#pragma unroll
                    for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                        const int bb = t + q * C::T;
                        if (!(I::even(I::S - 1) || bb < NBL)) continue;
#pragma unroll
                        for (int r0 = 0; r0 < RL; r0 += SCH) {
                            float2 s1[SCH], s2[SCH];
#pragma unroll
                            for (int i = 0; i < SCH; ++i) {
                                const int m = bb + (r0 + i) * NBL;
                                s1[i] = s2[i] = c_make(0.f, 0.f);
                                if (!fresh) {
                                    if (rvs && 2 * m + 1 < out_cols) {
                                        if constexpr (with_sum) s1[i] = reinterpret_cast<const float2*>(srow)[m];
                                        s2[i] = reinterpret_cast<const float2*>(qrow)[m];
                                    } else {
                                        if (2 * m < out_cols) {
                                            if constexpr (with_sum) s1[i].x = srow[2 * m];
                                            s2[i].x = qrow[2 * m];
                                        }
                                        if (2 * m + 1 < out_cols) {
                                            if constexpr (with_sum) s1[i].y = srow[2 * m + 1];
                                            s2[i].y = qrow[2 * m + 1];
                                        }
                                    }
                                }
                            }
#pragma unroll
                            for (int i = 0; i < SCH; ++i) {
                                const int m = bb + (r0 + i) * NBL;
                                const float2 z = v[q * RL + r0 + i];
                                const float2 a = c_make(s1[i].x + z.x, s1[i].y + z.y);
                                const float2 b2 =
                                    c_make(fmaf(z.x, z.x, s2[i].x), fmaf(z.y, z.y, s2[i].y));
                                if (rvs && 2 * m + 1 < out_cols) {
                                    if constexpr (with_sum) reinterpret_cast<float2*>(srow)[m] = a;
                                    reinterpret_cast<float2*>(qrow)[m] = b2;
                                } else {
                                    if (2 * m < out_cols) {
                                        if constexpr (with_sum) srow[2 * m] = a.x;
                                        qrow[2 * m] = b2.x;
                                    }
                                    if (2 * m + 1 < out_cols) {
                                        if constexpr (with_sum) srow[2 * m + 1] = a.y;
                                        qrow[2 * m + 1] = b2.y;
                                    }
                                }
                            }
                        }
                    }
                }
            }
        }
        // Rows past the end contribute -inf.
        if constexpr (MODE == kStorePeak) pk_run = fmax_nan(pk_run, pk);
        tj = next_tj;
        grp = next_grp;
        have = more;
    }
    if constexpr (MODE == kStorePeak) {
        if (pk_t >= 0) fold_block_peak(pk_run, peak + pk_t, red);
    }
}

// ===========================================================================
// Kernel 3, row-pair form (the map epilogues).  The two real rows y0, y1 of a
// pair come out of ONE W-point complex inverse FFT of Z = X_y0 + i X_y1, both
// spectra extended by Hermitian symmetry (X[W - k] = conj X[k]) from the
// packed tile: out[y0] = Re z, out[y1] = Im z.  This replaces the split
// pre-pass of the W/2-point form (one 16-byte read and two adds per element
// instead of two reads and two complex products).  Same tiles, tensor map and
// block size as k_row_c2r: a pair's W-point transform has twice the threads
// of a row's W/2-point one.
// ===========================================================================
template <int W2>
struct C2rPairCfg {
    using C = C2rCfg<W2>;
    static constexpr int W = 2 * W2;
    static constexpr int TP = fft_threads(W);  // threads per pair
    static constexpr int PPB = C::RPB / 2;     // pairs per block
    static constexpr int XB = xbuf_len(W);
    static constexpr int FLOATS = 2 * C::QB + PPB * XB;
    static constexpr int SMEM = FLOATS * 8 + 2 * 8 + 32 * 4;  // as C2rCfg
    static_assert(PPB * TP == C::THREADS, "a pair's transform has twice a row's threads");
};

template <int W2, int MODE>
__global__ void __launch_bounds__(C2rCfg<W2>::THREADS, C2rCfg<W2>::MINB)
    k_row_c2r_pair(const __grid_constant__ CUtensorMap qmap, float* __restrict__ out,
                   unsigned* __restrict__ peak, const float4* __restrict__ twt, int out_rows,
                   int out_cols, int out_pitch, int ntemplates, long long out_tstride,
                   int* __restrict__ status) {
    static_assert(MODE == kStoreMap || MODE == kStorePeak, "map epilogues only");
    using C = C2rCfg<W2>;
    using P = C2rPairCfg<W2>;
    constexpr int W = P::W, TP = P::TP;
    using I = Stockham<W, TP, true, false>;
    static_assert(I::S >= 2, "row FFT needs at least two stages");
    constexpr int R0 = I::radix(0), NB0 = I::nbf(0);
    constexpr int RL = I::radix(I::S - 1), NBL = I::nbf(I::S - 1);

    const int tid = threadIdx.x;
    const int pr = tid / TP, t = tid % TP;
    float2* smem = dyn_smem();
    float2* qbase = smem;  // [2][W2][RPB]
    float2* xbuf = smem + 2 * C::QB + pr * P::XB;
    uint64_t* mbar = reinterpret_cast<uint64_t*>(smem + P::FLOATS);
    float* red = reinterpret_cast<float*>(mbar + 2);  // kStorePeak's block reduction

    if (tid == 0) {
        mbar_init(&mbar[0], 1);
        mbar_init(&mbar[1], 1);
        mbar_init_fence();
    }
    __syncthreads();

    pdl_launch_dependents();
    typename I::Twiddles tw;
    I::load_thread_twiddles(tw, twt, t);
    // Q comes from the previous kernel.
    pdl_wait_prerequisites();

    // Units (template, row group) as in k_row_c2r.
    const int ngroups = (out_rows + C::RPB - 1) / C::RPB;
    const int units = ngroups * ntemplates;
    const uint64_t pol_keep = l2_evict_last();
    const uint64_t pol_stream = l2_evict_first();
    auto issue = [&](int b, int u) {
        const int tj = u / ngroups, grp = u - tj * ngroups;
        mbar_arrive_expect_tx(&mbar[b], (uint32_t)(W2 * C::RPB * 8));
        for (int k0 = 0; k0 < W2; k0 += C::BOXK)
            tma_load_2d(qbase + b * C::QB + k0 * C::RPB, &qmap, grp * C::RPB, tj * W2 + k0,
                        &mbar[b], pol_keep);
    };

    int u = blockIdx.x;
    if (tid == 0 && u < units) issue(0, u);
    float pk_run = -INFINITY;  // kStorePeak: this thread's largest value of template pk_t so far
    int pk_t = -1;
    for (int it = 0; u < units; ++it, u += gridDim.x) {
        const int tj = u / ngroups, grp = u - tj * ngroups;
        float* outj = out + tj * out_tstride;
        if constexpr (MODE == kStorePeak) {
            if (pk_t >= 0 && pk_t != tj) {  // block-uniform
                fold_block_peak(pk_run, peak + pk_t, red);
                pk_run = -INFINITY;
            }
            pk_t = tj;
        }
        const int b = it & 1;
        const uint32_t parity = (it >> 1) & 1;
        const bool more = u + (int)gridDim.x < units;
        if (tid == 0 && more) issue(b ^ 1, u + gridDim.x);
        const bool ok = mbar_wait_bounded(&mbar[b], parity);
        if (__syncthreads_or(!ok)) {  // block-uniform: every lane folds its warp
            if constexpr (MODE == kStorePeak) {
                if (pk_t >= 0) fold_block_peak(pk_run, peak + pk_t, red);
            }
            if (tid == 0) {
                atomicExch(status, kStatusTimeout);
                if (more) mbar_wait_bounded(&mbar[b ^ 1], ((it + 1) >> 1) & 1);
            }
            return;
        }

        // Stage-0 inputs Z[k], k = bb + r NB0: for k <= W2 from column k of the
        // tile, above from column W - k (conjugated); both rows of the pair in
        // one 16-byte read (X0.x, X0.y, X1.x, X1.y).  Packed column 0 holds
        // X[0] (real part) and X[W2] (imaginary part).  A second row past the
        // output (odd out_rows) was never written by the column pass: it
        // enters as zero, so that its stale contents cannot leak into the
        // first row through rounding (or as NaN).
        const int y0 = grp * C::RPB + 2 * pr;
        const bool has0 = y0 < out_rows, has1 = y0 + 1 < out_rows;
        const float2* qt = qbase + b * C::QB + 2 * pr;
        float2 v[I::MAXE];
#pragma unroll
        for (int q = 0; q < I::bpt(0); ++q) {
            const int bb = t + q * TP;
            if (I::even(0) || bb < NB0) {
#pragma unroll
                for (int r = 0; r < R0; ++r) {
                    const int k = bb + r * NB0;
                    const bool hi = k > W2;
                    const int j = hi ? W - k : k;
                    const int jt = j == W2 ? 0 : j;
                    float4 x = *reinterpret_cast<const float4*>(qt + jt * C::RPB);
                    if (!has1) x.z = x.w = 0.f;
                    float2 z;
                    if (j == 0)
                        z = c_make(x.x, x.z);
                    else if (j == W2)
                        z = c_make(x.y, x.w);
                    else if (!hi)
                        z = c_make(x.x - x.w, x.y + x.z);  // X0 + i X1
                    else
                        z = c_make(x.x + x.w, x.z - x.y);  // conj X0 + i conj X1
                    v[q * R0 + r] = z;
                }
            }
        }
        // No barrier after the last exchange: the epilogue uses registers and
        // global memory only, and the next group's first write of the
        // exchange buffer is behind the loop-top barrier.
        I::template run_regs<false>(v, xbuf, tw, t);

        // z[n] = out[y0][n] + i out[y1][n], n = bb + r NBL.
        float* row0 = outj + (size_t)y0 * out_pitch;
        float* row1 = row0 + out_pitch;
        float pk = -INFINITY;
        auto emit = [&](auto full_width) {
            constexpr bool FULL = decltype(full_width)::value;
#pragma unroll
            for (int q = 0; q < I::bpt(I::S - 1); ++q) {
                const int bb = t + q * TP;
                if (I::even(I::S - 1) || bb < NBL) {
#pragma unroll
                    for (int r = 0; r < RL; ++r) {
                        const int n = bb + r * NBL;
                        const float2 z = v[q * RL + r];
                        if (FULL || n < out_cols) {
                            if (has0) {
                                st_hint(row0 + n, z.x, pol_stream);
                                if constexpr (MODE == kStorePeak) pk = fmax_nan(pk, z.x);
                            }
                            if (has1) {
                                st_hint(row1 + n, z.y, pol_stream);
                                if constexpr (MODE == kStorePeak) pk = fmax_nan(pk, z.y);
                            }
                        }
                    }
                }
            }
        };
        if (out_cols == W)
            emit(std::true_type{});
        else
            emit(std::false_type{});
        if constexpr (MODE == kStorePeak) pk_run = fmax_nan(pk_run, pk);
    }
    if constexpr (MODE == kStorePeak) {
        if (pk_t >= 0) fold_block_peak(pk_run, peak + pk_t, red);
    }
}

}  // namespace zf
