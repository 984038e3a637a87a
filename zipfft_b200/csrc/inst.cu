// Kernel instantiations and launchers for one FFT size.  Compiled once per
// size with -DZF_SIZE=<n> (the build runs these compilations in parallel); each
// object defines launch_row_r2c_<n>, launch_col_<n>, make_qmap_<n> and
// launch_row_c2r_<n>.
//
// Replaces the per-configuration template instantiation of zipFFT's launcher
// (src/cuda/real_conv_2d.cuh:153-293 and the compile-time shape table in
// src/cuda/real_conv_2d_binding.cu:51-140): shapes other than the FFT size are
// run-time values here.
#include <mutex>
#include <utility>

#include "launch.h"
#include "xcorr_kernels.cuh"

#ifndef ZF_SIZE
#error "compile once per FFT size with -DZF_SIZE=<n>"
#endif

namespace zf {
namespace {

constexpr int kMaxDevices = 64;

// Per kernel instance and device: dynamic shared memory opt-in and the number
// of co-resident blocks, computed once.
struct KernelState {
    std::once_flag once[kMaxDevices];
    int grid_cap[kMaxDevices];
    cudaError_t err[kMaxDevices];
};

template <class Kern>
cudaError_t configure(Kern kernel, KernelState& st, int smem, int threads, int device, int* cap) {
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    std::call_once(st.once[device], [&] {
        cudaError_t e = cudaSuccess;
        if (smem > 48 * 1024)
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        int occ = 0, sms = 0;
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
        st.err[device] = e;
        st.grid_cap[device] = occ * sms;
    });
    *cap = st.grid_cap[device];
    if (st.err[device] != cudaSuccess) return st.err[device];
    return *cap > 0 ? cudaSuccess : cudaErrorInvalidConfiguration;
}

inline int min_int(int a, int b) { return a < b ? a : b; }

// Per-thread twiddle tables of this size's kernels (Stockham::fill_thread_twiddles),
// filled once per device by init_thread_twiddles_<n> from the size's root table:
//   row: the W/2-point plan of the row kernels (k_row_r2c, k_row_c2r);
//   col: the n-point plan (k_col_fused's forward transform, k_col_fwd, k_row_c2r_pair);
//   rev: the n-point plan reversed (k_col_fused's inverse when the plan is not a palindrome).
using RowPlan = Stockham<ZF_SIZE / 2, fft_threads(ZF_SIZE / 2), false, false>;
using ColPlan = Stockham<ZF_SIZE, fft_threads(ZF_SIZE), false, false>;
using RevPlan = Stockham<ZF_SIZE, fft_threads(ZF_SIZE), true, true>;
__device__ float4 g_tt_row[RowPlan::TWU * RowPlan::kThreads];
__device__ float4 g_tt_col[ColPlan::TWU * ColPlan::kThreads];
__device__ float4 g_tt_rev[RevPlan::TWU * RevPlan::kThreads];
constexpr int kTtThreads = cmax(RowPlan::kThreads, ColPlan::kThreads);

__global__ void k_fill_thread_twiddles(const float2* __restrict__ roots) {
    const int t = threadIdx.x;
    if (blockIdx.x == 0 && t < RowPlan::kThreads)
        RowPlan::template fill_thread_twiddles<ZF_SIZE>(g_tt_row, roots, t);
    if (blockIdx.x == 1 && t < ColPlan::kThreads)
        ColPlan::template fill_thread_twiddles<ZF_SIZE>(g_tt_col, roots, t);
    if (blockIdx.x == 2 && t < RevPlan::kThreads)
        RevPlan::template fill_thread_twiddles<ZF_SIZE>(g_tt_rev, roots, t);
}

struct ThreadTwiddles {
    const float4* row = nullptr;
    const float4* col = nullptr;
    const float4* rev = nullptr;
};
ThreadTwiddles g_tt[kMaxDevices];  // device addresses, set by init_thread_twiddles

// Launch with (pdl) or without programmatic stream serialization: with it
// the kernel may start while the previous kernel of the stream finishes; it
// calls griddepcontrol.wait before touching that kernel's data (a no-op
// without the attribute).
template <class... KArgs, class... Args>
cudaError_t launch_ex(bool pdl, void (*kernel)(KArgs...), dim3 grid, int threads, int smem,
                      cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, int threads, int smem, cudaStream_t s,
                       Args&&... args) {
    return launch_ex(true, kernel, grid, threads, smem, s, std::forward<Args>(args)...);
}

template <int W2, int NZ>
cudaError_t r2c_t(const float* tmpl, float2* R, const float2* tw, int h, int w, int r_pitch,
                  long long r_tstride, int ntemplates, float scale, int device, cudaStream_t s) {
    using C = R2cCfg<W2>;
    static KernelState st;
    auto kernel = k_row_r2c<W2, NZ>;
    int cap = 0;
    cudaError_t e = configure(kernel, st, C::SMEM, C::THREADS, device, &cap);
    if (e != cudaSuccess) return e;
    // One wave of co-resident blocks over all (template, row group) pairs.
    const long long units = (long long)((h + 1) / 2 * 2 + C::RPB - 1) / C::RPB * ntemplates;
    const int grid = (int)(units < cap ? units : cap);
    return launch_pdl(kernel, dim3(grid > 0 ? grid : 1), C::THREADS, C::SMEM, s, tmpl, R, tw,
                      g_tt[device].row, h, w, r_pitch, r_tstride, ntemplates, scale);
}

template <int H, bool CONJ, int NZ>
cudaError_t col_t(float2* Q, const float2* R, int r_pitch, const float2* spec, const float2* tw,
                  int h, int W2, int store_rows, bool discard_r, int ntemplates,
                  long long q_tstride, long long r_tstride, int* status, int device,
                  cudaStream_t s) {
    using C = ColCfg<H, NZ>;
    static KernelState st;
    auto kernel = k_col_fused<H, CONJ, NZ>;
    int cap = 0;
    cudaError_t e = configure(kernel, st, C::SMEM, C::THREADS, device, &cap);
    if (e != cudaSuccess) return e;
    const long long units = (long long)((W2 + C::FPB) / C::FPB) * ntemplates;
    const int grid = (int)(units < cap ? units : cap);
    return launch_pdl(kernel, dim3(grid), C::THREADS, C::SMEM, s, Q, R, r_pitch, spec,
                      g_tt[device].col, g_tt[device].rev, h, W2, store_rows, discard_r ? 1 : 0,
                      ntemplates, q_tstride, r_tstride, status);
}

template <int H>
cudaError_t col_fwd_t(float2* spec, const float2* tw, int W2, int* status, int device,
                      cudaStream_t s) {
    using C = ColFwdCfg<H>;
    static KernelState st;
    auto kernel = k_col_fwd<H>;
    int cap = 0;
    cudaError_t e = configure(kernel, st, C::SMEM, C::THREADS, device, &cap);
    if (e != cudaSuccess) return e;
    const int grid = min_int((W2 + C::FPB - 1) / C::FPB, cap);
    return launch_pdl(kernel, dim3(grid), C::THREADS, C::SMEM, s, spec, g_tt[device].col, W2,
                      status);
}

template <int W2, int MODE>
cudaError_t c2r_t(const CUtensorMap* qmap, float* out, int* arg, float* sum, float* sumsq,
                  unsigned* peak, const float2* tw, int out_rows, int out_cols, int out_pitch,
                  int tindex, int reset, int ntemplates, long long out_tstride, int* status,
                  int device, cudaStream_t s) {
    using C = C2rCfg<W2>;
    static KernelState st;
    auto kernel = k_row_c2r<W2, MODE>;
    int cap = 0;
    cudaError_t e = configure(kernel, st, C::SMEM, C::THREADS, device, &cap);
    if (e != cudaSuccess) return e;
    // The running-map modes hand each block whole row groups (all of the
    // launch's templates for each), the map modes (template, group) units.
    const long long groups = (out_rows + C::RPB - 1) / C::RPB;
    constexpr bool kRunning = MODE == kRunningMax || MODE == kRunningStats || MODE == kRunningSumSq;
    const long long units = kRunning ? groups : groups * ntemplates;
    const int grid = (int)(units < cap ? units : cap);
    // The peaks epilogue over a group of templates is launched without
    // programmatic serialization: with it, the launch ran 1.2-1.4x longer and
    // varied from call to call (measured at 4096^2 / 32 x 256^2; without its
    // atomics, or without the attribute, it matches the maps epilogue).
    const bool pdl = !(MODE == kStorePeak && ntemplates > 1);
    return launch_ex(pdl, kernel, dim3(grid), C::THREADS, C::SMEM, s, *qmap, out, arg, sum, sumsq,
                     peak, tw, g_tt[device].row, out_rows, out_cols, out_pitch, tindex, reset,
                     ntemplates, out_tstride, status);
}

template <int W2, int MODE>
cudaError_t c2r_pair_t(const CUtensorMap* qmap, float* out, unsigned* peak, const float2* tw,
                       int out_rows, int out_cols, int out_pitch, int ntemplates,
                       long long out_tstride, int* status, int device, cudaStream_t s) {
    using C = C2rCfg<W2>;
    using P = C2rPairCfg<W2>;
    static KernelState st;
    auto kernel = k_row_c2r_pair<W2, MODE>;
    int cap = 0;
    cudaError_t e = configure(kernel, st, P::SMEM, C::THREADS, device, &cap);
    if (e != cudaSuccess) return e;
    const long long units = (long long)((out_rows + C::RPB - 1) / C::RPB) * ntemplates;
    const int grid = (int)(units < cap ? units : cap);
    const bool pdl = !(MODE == kStorePeak && ntemplates > 1);  // as c2r_t
    return launch_ex(pdl, kernel, dim3(grid), C::THREADS, P::SMEM, s, *qmap, out, peak,
                     g_tt[device].col, out_rows, out_cols, out_pitch, ntemplates, out_tstride,
                     status);
}

// The pruned starts (nz = 1, 2) are instantiated for sizes >= 1024, where
// templates are much smaller than the image; smaller sizes use the full start.
constexpr bool kPruned = ZF_SIZE >= 1024;

}  // namespace

#define ZF_CAT2(a, b) a##b
#define ZF_CAT(a, b) ZF_CAT2(a, b)

cudaError_t ZF_CAT(init_thread_twiddles_, ZF_SIZE)(const float2* roots, int device) {
    if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
    k_fill_thread_twiddles<<<3, kTtThreads>>>(roots);
    cudaError_t e = cudaGetLastError();
    void* p = nullptr;
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_tt_row);
    if (e != cudaSuccess) return e;
    g_tt[device].row = static_cast<const float4*>(p);
    if ((e = cudaGetSymbolAddress(&p, g_tt_col)) != cudaSuccess) return e;
    g_tt[device].col = static_cast<const float4*>(p);
    if ((e = cudaGetSymbolAddress(&p, g_tt_rev)) != cudaSuccess) return e;
    g_tt[device].rev = static_cast<const float4*>(p);
    return cudaSuccess;
}

cudaError_t ZF_CAT(launch_row_r2c_, ZF_SIZE)(const float* tmpl, float2* R, const float2* tw, int h,
                                             int w, int r_pitch, long long r_tstride,
                                             int ntemplates, float scale, int nz, int device,
                                             cudaStream_t s) {
    constexpr int W2 = ZF_SIZE / 2;
    if constexpr (kPruned) {
        if (nz == 1) return r2c_t<W2, 1>(tmpl, R, tw, h, w, r_pitch, r_tstride, ntemplates, scale, device, s);
        if (nz == 2) return r2c_t<W2, 2>(tmpl, R, tw, h, w, r_pitch, r_tstride, ntemplates, scale, device, s);
    }
    return r2c_t<W2, 0>(tmpl, R, tw, h, w, r_pitch, r_tstride, ntemplates, scale, device, s);
}

cudaError_t ZF_CAT(launch_col_, ZF_SIZE)(float2* Q, const float2* R, int r_pitch,
                                         const float2* spec, const float2* tw, int h, int W2,
                                         int store_rows, bool conj, int nz, bool discard_r,
                                         int ntemplates, long long q_tstride, long long r_tstride,
                                         int* status, int device, cudaStream_t s) {
    constexpr int H = ZF_SIZE;
#define ZF_COL(CJ, NZV)                                                                       \
    col_t<H, CJ, NZV>(Q, R, r_pitch, spec, tw, h, W2, store_rows, discard_r, ntemplates,      \
                      q_tstride, r_tstride, status, device, s)
    if constexpr (kPruned) {
        if (nz == 1) return conj ? ZF_COL(true, 1) : ZF_COL(false, 1);
        if (nz == 2) return conj ? ZF_COL(true, 2) : ZF_COL(false, 2);
    }
    return conj ? ZF_COL(true, 0) : ZF_COL(false, 0);
#undef ZF_COL
}

cudaError_t ZF_CAT(launch_col_fwd_, ZF_SIZE)(float2* spec, const float2* tw, int W2, int* status,
                                             int device, cudaStream_t s) {
    return col_fwd_t<ZF_SIZE>(spec, tw, W2, status, device, s);
}

cudaError_t ZF_CAT(make_qmap_, ZF_SIZE)(const float2* Q, int H, int ntemplates, CUtensorMap* map) {
    using C = C2rCfg<ZF_SIZE / 2>;
    // Q is column-major: dim 0 = rows y (H, contiguous), dim 1 = packed columns
    // of ntemplates consecutive slices.
    return encode_tensor_map_2d(map, Q, (unsigned long long)H,
                                (unsigned long long)(ZF_SIZE / 2) * (unsigned long long)ntemplates,
                                (unsigned long long)H * 8ull, C::RPB, C::BOXK);
}

cudaError_t ZF_CAT(launch_row_c2r_, ZF_SIZE)(const CUtensorMap* qmap, float* out, int* arg,
                                             float* sum, float* sumsq, unsigned* peak,
                                             const float2* tw, int out_rows, int out_cols,
                                             int out_pitch, int tindex, int reset, int ntemplates,
                                             long long out_tstride, int* status, int device,
                                             cudaStream_t s) {
    constexpr int W2 = ZF_SIZE / 2;
    if (ntemplates < 1) return cudaErrorInvalidValue;
    // Running maps: ntemplates consecutive templates (indices tindex, ...)
    // folded into the same maps (out_tstride unused).
    if (arg != nullptr && sum != nullptr && sumsq != nullptr)
        return c2r_t<W2, kRunningStats>(qmap, out, arg, sum, sumsq, nullptr, tw, out_rows,
                                        out_cols, out_pitch, tindex, reset, ntemplates, 0, status,
                                        device, s);
    if (arg != nullptr && sumsq != nullptr)  // the sum of squares alone
        return c2r_t<W2, kRunningSumSq>(qmap, out, arg, nullptr, sumsq, nullptr, tw, out_rows,
                                        out_cols, out_pitch, tindex, reset, ntemplates, 0, status,
                                        device, s);
    if (arg != nullptr)
        return c2r_t<W2, kRunningMax>(qmap, out, arg, nullptr, nullptr, nullptr, tw, out_rows,
                                      out_cols, out_pitch, tindex, reset, ntemplates, 0, status,
                                      device, s);
    // Maps.  Full-width rows that are all 8-byte aligned: the W/2-point form,
    // whose epilogue writes each output pair with one 8-byte store.  Cropped
    // or misaligned rows (the reference's valid crop, e.g. 3841 wide): the
    // row-pair form, which needs no split pre-pass and stores 4-byte values
    // anyway (measured: 13.6k against 13.0k corr/s for the 3841^2 crop of
    // 4096^2 / 256^2, and 13.4k against 13.6k for full maps).
    const bool full_aligned = out_cols == 2 * W2 && (out_pitch % 2) == 0 &&
                              (reinterpret_cast<size_t>(out) % 8) == 0 &&
                              (out_tstride % 2) == 0;
    if (full_aligned) {
        if (peak != nullptr)
            return c2r_t<W2, kStorePeak>(qmap, out, nullptr, nullptr, nullptr, peak, tw, out_rows,
                                         out_cols, out_pitch, 0, 0, ntemplates, out_tstride,
                                         status, device, s);
        return c2r_t<W2, kStoreMap>(qmap, out, nullptr, nullptr, nullptr, nullptr, tw, out_rows,
                                    out_cols, out_pitch, 0, 0, ntemplates, out_tstride, status,
                                    device, s);
    }
    if (peak != nullptr)
        return c2r_pair_t<W2, kStorePeak>(qmap, out, peak, tw, out_rows, out_cols, out_pitch,
                                          ntemplates, out_tstride, status, device, s);
    return c2r_pair_t<W2, kStoreMap>(qmap, out, nullptr, tw, out_rows, out_cols, out_pitch,
                                     ntemplates, out_tstride, status, device, s);
}

}  // namespace zf
