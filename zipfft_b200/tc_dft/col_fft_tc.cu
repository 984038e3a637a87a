// Radix-16 FFT stages on the tensor cores (tcgen05.mma, kind::tf32) against
// the same stages on the CUDA cores: a measured A/B for the column FFTs of the
// correlation pipeline (the cuFFTDx block FFTs that zipFFT calls at
// src/cuda/real_conv_2d.cuh:84,114).  Not on the product path.
//
// Both kernels run the same in-place 4096-point forward complex FFT over
// `columns` contiguous columns -- the column pass of the image spectrum, 2049
// columns of 4096 points for a 4096^2 image -- as three radix-16 stages
// (n = m + 256 n2, m = n0 + 16 n1; Cooley-Tukey with the twiddles between
// stages), with the same loads, twiddle tables, shared-memory rows and
// stores.  They differ only in how each thread's 16-point DFT is computed:
//
//   * CUDA cores: zf::dft16 on the thread's 16 values in registers;
//   * tensor cores: the block's 256 rows of 16 complex values are the A
//     operand of a (256 x 32) x (32 x 32) real GEMM against the 16-point DFT
//     matrix written as real 2 x 2 blocks, on tcgen05.mma kind::tf32 with the
//     3-pass split x = x_hi + x_lo (x_hi rounded to TF32):
//     A_hi B_hi + A_hi B_lo + A_lo B_hi, accumulated in TMEM (fp32) and read
//     back by tcgen05.ld, one TMEM lane (= one row) per thread.
//
// Shared-memory rows are 128 bytes (16 complex float) in the 128-byte-swizzle
// K-major layout the tensor core reads: 16-byte chunk c of row r sits at
// chunk position c ^ (r & 7) of the row, rows contiguous, 1024-byte atoms.
// The CUDA-core kernel uses the same layout for its exchanges, which keeps
// every exchange free of bank conflicts in both kernels.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <vector>

#include "../csrc/async_copy.cuh"
#include "../csrc/fft_core.cuh"

namespace zftc {

constexpr int kN = 4096;
constexpr int kT = 256;                         // threads per block = rows per stage
constexpr int kRowBytes = 128;                  // 16 complex float
constexpr int kABytes = kT * kRowBytes;         // one copy of the A operand: 32 KB
constexpr int kBBytes = 32 * kRowBytes;         // one copy of the DFT matrix: 4 KB
constexpr int kTmemCols = 64;                   // two 128-row halves x 32 fp32 columns
// Shared memory: [A_hi | A_lo | B_hi | B_lo | mbarrier, TMEM slot], 1024-aligned.
constexpr int kSmemTc = 2 * kABytes + 2 * kBBytes + 64 + 1024;
constexpr int kSmemCuda = kABytes + 1024;

// Instruction descriptor, kind::tf32: D fp32 (bits 4-5 = 1), A and B TF32
// (bits 7-9, 10-12 = 2), both K-major (bits 15, 16 = 0), N = 32 (bits 17-22:
// N >> 3), M = 128 (bits 24-28: M >> 4).
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((32u >> 3) << 17) |
                            ((128u >> 4) << 24);

ZF_DEV uint32_t row_off(int row, int chunk) {
    return uint32_t(row * kRowBytes + ((chunk ^ (row & 7)) << 4));
}

// Shared-memory matrix descriptor: 128-byte swizzle (layout 2, bits 61-63),
// K-major canonical layout with 8-row atoms of 1024 bytes (stride byte offset
// 1024, bits 32-45), leading byte offset unused for this layout (16 bytes),
// descriptor version 1 (bit 46), start address >> 4 in bits 0-13.
ZF_DEV uint64_t smem_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3FFFu);
    d |= uint64_t(16 >> 4) << 16;
    d |= uint64_t(1024 >> 4) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

ZF_DEV float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

ZF_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ZF_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

ZF_DEV void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        :
        : "r"(tmem_d), "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

ZF_DEV void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     zf::smem_u32(bar))
                 : "memory");
}

// 32 consecutive fp32 TMEM columns of this thread's lane.
ZF_DEV void tc_ld32(uint32_t taddr, float2* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = make_float2(__uint_as_float(r[2 * k]), __uint_as_float(r[2 * k + 1]));
}

// A row of 16 complex values, split into its TF32 part and the remainder.
ZF_DEV void write_row_split(unsigned char* hi, unsigned char* lo, int row, const float2* v) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float4 x = make_float4(v[2 * c].x, v[2 * c].y, v[2 * c + 1].x, v[2 * c + 1].y);
        const float4 h = make_float4(tf32_round(x.x), tf32_round(x.y), tf32_round(x.z), tf32_round(x.w));
        const uint32_t o = row_off(row, c);
        *reinterpret_cast<float4*>(hi + o) = h;
        *reinterpret_cast<float4*>(lo + o) = make_float4(x.x - h.x, x.y - h.y, x.z - h.z, x.w - h.w);
    }
}

// One complex value at position `pos` of a row, split like write_row_split.
ZF_DEV void write_pos_split(unsigned char* hi, unsigned char* lo, int row, int pos, float2 x) {
    const float2 h = make_float2(tf32_round(x.x), tf32_round(x.y));
    const uint32_t o = row_off(row, pos >> 1) + uint32_t(pos & 1) * 8;
    *reinterpret_cast<float2*>(hi + o) = h;
    *reinterpret_cast<float2*>(lo + o) = make_float2(x.x - h.x, x.y - h.y);
}

ZF_DEV void write_pos(unsigned char* buf, int row, int pos, float2 x) {
    *reinterpret_cast<float2*>(buf + row_off(row, pos >> 1) + uint32_t(pos & 1) * 8) = x;
}

ZF_DEV void read_row(const unsigned char* buf, int row, float2* v) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        const float4 q = *reinterpret_cast<const float4*>(buf + row_off(row, c));
        v[2 * c] = make_float2(q.x, q.y);
        v[2 * c + 1] = make_float2(q.z, q.w);
    }
}

// In-place forward 4096-point FFT of `columns` contiguous columns, applied
// `passes` times to each column between its load and its store (2 passes do
// twice the arithmetic per byte, like the fused column pass's forward and
// inverse transforms); one block per column at a time (persistent grid).  tw1[k * 256 + t] = W_4096^(t k),
// tw2[k * 256 + t] = W_256^((t mod 16) k) (thread t's twiddles, coalesced);
// bmat: the 32 x 32 real DFT-16 matrix, row n of B = column n of the GEMM
// (K-major), used by the tensor-core kernel only.
template <bool TC>
__global__ void __launch_bounds__(kT) k_col_fft4096(float2* __restrict__ data, int columns,
                                                    int passes,
                                                    const float2* __restrict__ tw1,
                                                    const float2* __restrict__ tw2,
                                                    const float* __restrict__ bmat,
                                                    int* __restrict__ status) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = zf::smem_u32(smem_raw);
    unsigned char* base = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    unsigned char* a_hi = base;
    unsigned char* a_lo = base + kABytes;
    unsigned char* b_hi = base + 2 * kABytes;
    unsigned char* b_lo = b_hi + kBBytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(b_lo + kBBytes);
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar + 1);
    const int t = threadIdx.x, warp = t >> 5;

    uint32_t tmem = 0;
    if constexpr (TC) {
        for (int i = t; i < 32 * 32; i += kT) {
            const int r = i >> 5, k = i & 31;
            const float b = bmat[i];
            const float h = tf32_round(b);
            *reinterpret_cast<float*>(b_hi + row_off(r, k >> 2) + (k & 3) * 4) = h;
            *reinterpret_cast<float*>(b_lo + row_off(r, k >> 2) + (k & 3) * 4) = b - h;
        }
        if (t == 0) {
            zf::mbar_init(bar, 1);
            zf::mbar_init_fence();
        }
        if (warp == 0) {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             zf::smem_u32(tslot)),
                         "r"(kTmemCols)
                         : "memory");
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        }
        zf::fence_proxy_async();  // the DFT matrix is read by the tensor core's (async) proxy
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        tmem = *tslot;
    }
    // This thread's TMEM lane (= its row) and column half.
    const uint32_t tmem_row = tmem + ((uint32_t(warp & 3) * 32u) << 16) + uint32_t(warp >> 2) * 32u;

    uint32_t phase = 0;
    bool failed = false;
    // The block's 256 rows (A, split) times the DFT matrix; each thread gets
    // its own row's 16 outputs back in v.
    auto mma_round = [&](float2* v) {
        zf::fence_proxy_async();
        tc_fence_before();
        __syncthreads();
        if (t == 0) {
            tc_fence_after();
            const uint64_t bh = smem_desc(zf::smem_u32(b_hi)), bl = smem_desc(zf::smem_u32(b_lo));
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint64_t ah = smem_desc(zf::smem_u32(a_hi + h * (kABytes / 2)));
                const uint64_t al = smem_desc(zf::smem_u32(a_lo + h * (kABytes / 2)));
                const uint32_t d = tmem + uint32_t(h) * 32u;
                // K = 32 floats per row = 4 steps of 8 (32 bytes: +2 in the
                // descriptor's start-address field).
#pragma unroll
                for (int k = 0; k < 4; ++k) tc_mma(d, ah + 2 * k, bh + 2 * k, k > 0 ? 1u : 0u);
#pragma unroll
                for (int k = 0; k < 4; ++k) tc_mma(d, ah + 2 * k, bl + 2 * k, 1u);
#pragma unroll
                for (int k = 0; k < 4; ++k) tc_mma(d, al + 2 * k, bh + 2 * k, 1u);
            }
            tc_commit(bar);
        }
        if (!zf::mbar_wait_bounded(bar, phase)) failed = true;
        phase ^= 1u;
        __syncwarp();  // tcgen05.ld is warp-collective (.sync.aligned)
        tc_fence_after();
        tc_ld32(tmem_row, v);
    };

    for (int col = blockIdx.x; col < columns; col += gridDim.x) {
        float2* x = data + size_t(col) * kN;
        float2 v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = x[t + kT * j];
#pragma unroll 1
        for (int pass = 0; pass < passes; ++pass) {
            // Stage 1: row m = t holds x[m + 256 n2] at position n2.
            if constexpr (TC) {
                write_row_split(a_hi, a_lo, t, v);
                mma_round(v);
            } else {
                zf::dft16<false>(v);
            }
#pragma unroll
            for (int k = 1; k < 16; ++k) v[k] = zf::c_mul(v[k], tw1[k * kT + t]);
            // Stage 2: value k0 of row m = n0 + 16 n1 goes to row 16 k0 + n0,
            // position n1.
            const int n0 = t & 15, n1 = t >> 4;
            if constexpr (TC) {
#pragma unroll
                for (int k = 0; k < 16; ++k) write_pos_split(a_hi, a_lo, k * 16 + n0, n1, v[k]);
                mma_round(v);
            } else {
                __syncthreads();  // earlier reads of the buffer are done
#pragma unroll
                for (int k = 0; k < 16; ++k) write_pos(a_hi, k * 16 + n0, n1, v[k]);
                __syncthreads();
                read_row(a_hi, t, v);
                zf::dft16<false>(v);
            }
            // Row t = 16 k0 + n0 holds value k1: twiddle W_256^(n0 k1).
#pragma unroll
            for (int k = 1; k < 16; ++k) v[k] = zf::c_mul(v[k], tw2[k * kT + t]);
            // Stage 3: value k1 of row 16 k0 + n0 goes to row 16 k1 + k0,
            // position n0.
            if constexpr (TC) {
#pragma unroll
                for (int k = 0; k < 16; ++k) write_pos_split(a_hi, a_lo, k * 16 + n1, n0, v[k]);
                mma_round(v);
            } else {
                __syncthreads();
#pragma unroll
                for (int k = 0; k < 16; ++k) write_pos(a_hi, k * 16 + n1, n0, v[k]);
                __syncthreads();
                read_row(a_hi, t, v);
                zf::dft16<false>(v);
            }
            // Row t = 16 k1 + k0 holds X[k0 + 16 k1 + 256 k2] = X[t + 256 k2] at k2:
            // the layout of the input, so another pass can follow directly.
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) x[t + kT * j] = v[j];
        if constexpr (TC) {
            if (__syncthreads_or(failed)) break;
        }
    }

    if constexpr (TC) {
        if (failed) atomicOr(status, zf::kStatusTimeout);
        if (__syncthreads_or(failed) && t == 0) zf::mbar_wait_bounded(bar, phase ^ 1u);
        tc_fence_before();
        __syncthreads();
        if (warp == 0) {
            tc_fence_after();
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                         "r"(kTmemCols)
                         : "memory");
        }
    }
}

}  // namespace zftc

// ---------------------------------------------------------------------------
// C ABI (ctypes): zftc_col_fft4096 runs one of the two kernels.
// ---------------------------------------------------------------------------
#define ZFTC_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr int kMaxDev = 16;

struct DevState {
    bool ready = false;
    float2* tw1 = nullptr;
    float2* tw2 = nullptr;
    float* bmat = nullptr;
    int* status = nullptr;
    int sms = 0;
    int occ[2] = {0, 0};  // blocks per SM: CUDA-core kernel, tensor-core kernel
    int regs[2] = {0, 0};
};

DevState g_dev[kMaxDev];
std::mutex g_mu;
char g_err[512] = "";

int fail_cuda(const char* what, cudaError_t e) {
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return 1;
}

struct DeviceSwitch {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceSwitch(int dev) {
        err = cudaGetDevice(&prev);
        if (err == cudaSuccess && prev != dev) err = cudaSetDevice(dev);
    }
    ~DeviceSwitch() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// Host tables in double precision, rounded once to float.
void host_tables(std::vector<float2>& tw1, std::vector<float2>& tw2, std::vector<float>& bmat) {
    const double pi = 3.141592653589793238462643383279502884;
    tw1.resize(16 * zftc::kT);
    tw2.resize(16 * zftc::kT);
    for (int k = 0; k < 16; ++k)
        for (int t = 0; t < zftc::kT; ++t) {
            const double a1 = -2.0 * pi * double((t * k) % zftc::kN) / zftc::kN;
            const double a2 = -2.0 * pi * double(((t & 15) * k) % 256) / 256.0;
            tw1[k * zftc::kT + t] = make_float2(float(std::cos(a1)), float(std::sin(a1)));
            tw2[k * zftc::kT + t] = make_float2(float(std::cos(a2)), float(std::sin(a2)));
        }
    // Row 2k / 2k+1 of B: real / imaginary part of output k; column 2n / 2n+1:
    // real / imaginary part of input n.  X_k = sum_n x_n e^{-i theta},
    // theta = 2 pi n k / 16.
    bmat.assign(32 * 32, 0.0f);
    for (int k = 0; k < 16; ++k)
        for (int n = 0; n < 16; ++n) {
            const double th = 2.0 * pi * double((n * k) % 16) / 16.0;
            const float c = float(std::cos(th)), s = float(std::sin(th));
            bmat[(2 * k) * 32 + 2 * n] = c;
            bmat[(2 * k) * 32 + 2 * n + 1] = s;
            bmat[(2 * k + 1) * 32 + 2 * n] = -s;
            bmat[(2 * k + 1) * 32 + 2 * n + 1] = c;
        }
}

int ensure(int dev) {
    std::lock_guard<std::mutex> lock(g_mu);
    DevState& st = g_dev[dev];
    if (st.ready) return 0;
    std::vector<float2> tw1, tw2;
    std::vector<float> bmat;
    host_tables(tw1, tw2, bmat);
    cudaError_t e;
    if ((e = cudaMalloc(&st.tw1, tw1.size() * sizeof(float2))) != cudaSuccess) return fail_cuda("cudaMalloc", e);
    if ((e = cudaMalloc(&st.tw2, tw2.size() * sizeof(float2))) != cudaSuccess) return fail_cuda("cudaMalloc", e);
    if ((e = cudaMalloc(&st.bmat, bmat.size() * sizeof(float))) != cudaSuccess) return fail_cuda("cudaMalloc", e);
    if ((e = cudaMalloc(&st.status, sizeof(int))) != cudaSuccess) return fail_cuda("cudaMalloc", e);
    if ((e = cudaMemcpy(st.tw1, tw1.data(), tw1.size() * sizeof(float2), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(st.tw2, tw2.data(), tw2.size() * sizeof(float2), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(st.bmat, bmat.data(), bmat.size() * sizeof(float), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemset(st.status, 0, sizeof(int))) != cudaSuccess)
        return fail_cuda("table upload", e);
    if ((e = cudaFuncSetAttribute(zftc::k_col_fft4096<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  zftc::kSmemCuda)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zftc::k_col_fft4096<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  zftc::kSmemTc)) != cudaSuccess)
        return fail_cuda("cudaFuncSetAttribute", e);
    if ((e = cudaDeviceGetAttribute(&st.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
        return fail_cuda("cudaDeviceGetAttribute", e);
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&st.occ[0], zftc::k_col_fft4096<false>, zftc::kT,
                                                           zftc::kSmemCuda)) != cudaSuccess ||
        (e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&st.occ[1], zftc::k_col_fft4096<true>, zftc::kT,
                                                           zftc::kSmemTc)) != cudaSuccess)
        return fail_cuda("cudaOccupancyMaxActiveBlocksPerMultiprocessor", e);
    cudaFuncAttributes fa[2];
    if ((e = cudaFuncGetAttributes(&fa[0], zftc::k_col_fft4096<false>)) != cudaSuccess ||
        (e = cudaFuncGetAttributes(&fa[1], zftc::k_col_fft4096<true>)) != cudaSuccess)
        return fail_cuda("cudaFuncGetAttributes", e);
    st.regs[0] = fa[0].numRegs;
    st.regs[1] = fa[1].numRegs;
    // TMEM: every resident block of the tensor-core kernel holds kTmemCols of
    // the SM's 512 columns, so allocations never wait on one another.
    if (st.occ[1] * zftc::kTmemCols > 512) st.occ[1] = 512 / zftc::kTmemCols;
    st.ready = true;
    return 0;
}

}  // namespace

ZFTC_API const char* zftc_last_error() { return g_err; }

// In-place forward 4096-point FFTs of `columns` contiguous columns of complex64
// (column c at data + 4096 c), `passes` times each; tensor_cores selects the
// tcgen05 kernel; blocks_per_sm = 0 sizes the persistent grid by occupancy.
// Returns 0, or 1 with zftc_last_error() set.
ZFTC_API int zftc_col_fft4096(void* data, int columns, int passes, int tensor_cores, int blocks_per_sm,
                              int device, void* stream) {
    if (device < 0 || device >= kMaxDev) {
        snprintf(g_err, sizeof g_err, "invalid device %d", device);
        return 1;
    }
    if (columns < 0 || passes < 1 || blocks_per_sm < 0 || blocks_per_sm > 8 || (columns > 0 && !data) ||
        (reinterpret_cast<uintptr_t>(data) & 15u)) {
        snprintf(g_err, sizeof g_err, "invalid arguments");
        return 1;
    }
    DeviceSwitch sw(device);
    if (sw.err != cudaSuccess) return fail_cuda("cudaSetDevice", sw.err);
    if (ensure(device)) return 1;
    if (columns == 0) return 0;
    const DevState& st = g_dev[device];
    const int tc = tensor_cores ? 1 : 0;
    // blocks_per_sm > 0: launch that many blocks per SM instead of the
    // occupancy calculator's figure (the hardware runs the surplus as later
    // waves if they do not fit).
    int grid = st.sms * (blocks_per_sm > 0 ? blocks_per_sm : st.occ[tc]);
    if (grid > columns) grid = columns;
    if (grid < 1) {
        snprintf(g_err, sizeof g_err, "kernel does not fit on an SM");
        return 1;
    }
    auto s = static_cast<cudaStream_t>(stream);
    if (tc)
        zftc::k_col_fft4096<true><<<grid, zftc::kT, zftc::kSmemTc, s>>>(
            static_cast<float2*>(data), columns, passes, st.tw1, st.tw2, st.bmat, st.status);
    else
        zftc::k_col_fft4096<false><<<grid, zftc::kT, zftc::kSmemCuda, s>>>(
            static_cast<float2*>(data), columns, passes, st.tw1, st.tw2, st.bmat, st.status);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? 0 : fail_cuda("launch", e);
}

// Registers per thread and resident blocks per SM of one of the kernels.
ZFTC_API int zftc_kernel_info(int tensor_cores, int device, int* regs, int* blocks_per_sm) {
    if (device < 0 || device >= kMaxDev) return 1;
    DeviceSwitch sw(device);
    if (sw.err != cudaSuccess) return fail_cuda("cudaSetDevice", sw.err);
    if (ensure(device)) return 1;
    const int tc = tensor_cores ? 1 : 0;
    *regs = g_dev[device].regs[tc];
    *blocks_per_sm = g_dev[device].occ[tc];
    return 0;
}

// Resident blocks per SM of one kernel with `smem` bytes of dynamic shared
// memory, as the occupancy calculator reports it.
ZFTC_API int zftc_occupancy(int tensor_cores, int device, int smem, int* blocks_per_sm) {
    if (device < 0 || device >= kMaxDev) return 1;
    DeviceSwitch sw(device);
    if (sw.err != cudaSuccess) return fail_cuda("cudaSetDevice", sw.err);
    if (ensure(device)) return 1;
    const cudaError_t e =
        tensor_cores ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, zftc::k_col_fft4096<true>,
                                                                     zftc::kT, size_t(smem))
                     : cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks_per_sm, zftc::k_col_fft4096<false>,
                                                                     zftc::kT, size_t(smem));
    return e == cudaSuccess ? 0 : fail_cuda("occupancy", e);
}

// The device status word (4: a bounded wait gave up), then cleared.
ZFTC_API int zftc_status(int device, int* out) {
    if (device < 0 || device >= kMaxDev || !g_dev[device].ready) {
        *out = 0;
        return 0;
    }
    DeviceSwitch sw(device);
    if (sw.err != cudaSuccess) return fail_cuda("cudaSetDevice", sw.err);
    cudaError_t e = cudaMemcpy(out, g_dev[device].status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemset(g_dev[device].status, 0, sizeof(int));
    return e == cudaSuccess ? 0 : fail_cuda("status", e);
}
