// Internal launch entry points, one set per FFT size (defined in inst.cu,
// compiled once per size).  Not part of the public C ABI.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include "zf_sizes.h"

namespace zf {

// init_thread_twiddles_<n>: fills the per-thread twiddle tables of size n's
// kernels from the n-point root table on the current device (on the legacy
// default stream; the caller synchronizes) and records their addresses.  Every
// launcher of that size and device needs it first.
// Row r2c of `ntemplates` templates (h x w each, consecutive in tmpl) of a
// W-column image: R of template j at R + j * r_tstride, element (kx, n) at
// kx * r_pitch + n.  nz: 1 or 2 when the template row fits the first 1 or 2
// stage-0 inputs of every butterfly, else 0.
// Column pass of an H-row image: forward FFT of the h rows of R, product with
// the spectrum, inverse FFT, first store_rows rows of Q stored; ntemplates
// templates, template j's Q / R at Q + j q_tstride / R + j r_tstride.
// Image spectrum column pass: in place over the W2 packed columns (pitch H)
// that the row r2c wrote into spec, and the split of packed column 0 into
// rows 0 and W2.
// Row c2r: the Q tile map comes from make_qmap_<W> (same W, covering
// ntemplates consecutive Q slices); out_rows rows of out_cols values at
// out_pitch, template j's map at out + j out_tstride.  arg == nullptr: store the map into out;
// otherwise fold it into the running max (out) / argmax (arg) maps with
// template index tindex (reset: overwrite instead of compare), and with sum
// != nullptr also add it and its square to the sum / sumsq maps.  With
// arg == nullptr and peak != nullptr, the map's largest value is also folded
// into *peak as an ordered_key (atomicMax).
#define ZF_DECL(N)                                                                              \
    cudaError_t init_thread_twiddles_##N(const float2* roots, int device);                      \
    cudaError_t launch_row_r2c_##N(const float* tmpl, float2* R, const float2* tw, int h, int w, \
                                   int r_pitch, long long r_tstride, int ntemplates, float scale, \
                                   int nz, int device, cudaStream_t s);                          \
    cudaError_t launch_col_##N(float2* Q, const float2* R, int r_pitch, const float2* spec,      \
                               const float2* tw, int h, int W2, int store_rows, bool conj, int nz, \
                               bool discard_r, int ntemplates, long long q_tstride,              \
                               long long r_tstride, int* status, int device, cudaStream_t s);    \
    cudaError_t launch_col_fwd_##N(float2* spec, const float2* tw, int W2, int* status,         \
                                   int device, cudaStream_t s);                                  \
    cudaError_t make_qmap_##N(const float2* Q, int H, int ntemplates, CUtensorMap* map);        \
    cudaError_t launch_row_c2r_##N(const CUtensorMap* qmap, float* out, int* arg, float* sum,   \
                                   float* sumsq, unsigned* peak, const float2* tw, int out_rows, \
                                   int out_cols, int out_pitch, int tindex, int reset,           \
                                   int ntemplates, long long out_tstride, int* status,           \
                                   int device, cudaStream_t s);
ZF_FOR_EACH_FFT_SIZE(ZF_DECL)
#undef ZF_DECL

// First radix of the plan of an n-point transform (host side, for nz).
int plan_first_radix(int n);

// Encode a 2D tiled tensor map (driver entry point resolved once).
cudaError_t encode_tensor_map_2d(CUtensorMap* map, const void* base, unsigned long long dim0,
                                 unsigned long long dim1, unsigned long long stride1_bytes,
                                 unsigned box0, unsigned box1);

// Launch of the bounded-wait self-test kernel (capi.cu).
cudaError_t launch_wait_selftest(int* status, long long limit_cycles, cudaStream_t s);

}  // namespace zf
