// Internal launch entry points, one set per FFT size (defined in inst.cu,
// compiled once per size).  Not part of the public C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

#include "zf_sizes.h"

namespace zf {

// Column pass of an H-row image: forward FFT of the h non-zero rows of every
// packed column, product with the spectrum, inverse FFT, first store_rows rows
// stored in place.  nz: 1 or 2 when the non-zero rows fit the first 1 or 2
// stage-0 inputs of every butterfly, else 0.
#define ZF_DECL_COL(N)                                                                       \
    cudaError_t launch_col_##N(float2* ws, const float2* spec, const float2* tw, int h, int W2, \
                               int store_rows, bool conj, int nz, int device, cudaStream_t s);
// Row passes of a W-column image (FFT length W, folded to W/2 complex).
#define ZF_DECL_ROW(N)                                                                         \
    cudaError_t launch_row_r2c_##N(const float* tmpl, float2* ws, const float2* tw, int h,      \
                                   int w, int H, float scale, int nz, int device, cudaStream_t s); \
    cudaError_t launch_row_c2r_##N(const float2* ws, float* out, const float2* tw, int H,       \
                                   int out_rows, int out_cols, int out_pitch, int device,        \
                                   cudaStream_t s);
ZF_FOR_EACH_FFT_SIZE(ZF_DECL_COL)
ZF_FOR_EACH_FFT_SIZE(ZF_DECL_ROW)
#undef ZF_DECL_COL
#undef ZF_DECL_ROW

// First radix of the plan of an n-point transform (host side, for nz).
int plan_first_radix(int n);

}  // namespace zf
