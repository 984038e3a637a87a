// CPU execution of the library's CUDA kernels, for tests only.
//
// Each kernel block runs as blockDim std::threads sharing one shared-memory
// array and a std::barrier for __syncthreads; blocks run one after another.
// Built with AddressSanitizer, this checks the kernels' index arithmetic
// (every global and shared access in bounds) and their arithmetic against the
// oracle on small sizes before any of it runs on a GPU.  It is never part of
// the library: the library has no CPU path.
//
// Usage: zf_emu <in.bin> <out.bin>
//   in.bin : int32 header {B, sy, sx, H, W, oy, ox, conj, grid_cap, nz_col,
//            nz_row}, float32 templates [B][sy][sx], complex64 spectrum
//            [W/2+1][H]
//   out.bin: float32 [B][oy][ox]
#include <barrier>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <math.h>
#include <thread>
#include <vector>

struct float2 {
    float x, y;
};
struct dim3 {
    unsigned x = 1, y = 1, z = 1;
};
#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(...)

thread_local dim3 threadIdx, blockIdx, blockDim, gridDim;
thread_local std::barrier<>* emu_barrier = nullptr;
thread_local float2* emu_smem = nullptr;
inline void __syncthreads() { emu_barrier->arrive_and_wait(); }
template <class T>
inline T __ldg(const T* p) {
    return *p;
}

#include "../../zipfft_b200/csrc/xcorr_kernels.cuh"

float2* zf::dyn_smem() { return emu_smem; }

template <class K, class... A>
void emu_launch(int grid, int block, size_t smem_bytes, K kernel, A... args) {
    std::vector<float2> smem((smem_bytes + 7) / 8);
    std::barrier<> bar(block);
    std::vector<std::thread> threads;
    for (int tid = 0; tid < block; ++tid) {
        threads.emplace_back([&, tid] {
            threadIdx.x = tid;
            blockDim.x = block;
            gridDim.x = grid;
            emu_barrier = &bar;
            emu_smem = smem.data();
            for (int b = 0; b < grid; ++b) {
                blockIdx.x = b;
                kernel(args...);
                bar.arrive_and_wait();
            }
        });
    }
    for (auto& t : threads) t.join();
}

static std::vector<float2> twiddles(int n) {
    std::vector<float2> t(n);
    for (int m = 0; m < n; ++m) {
        double a = 2.0 * zf::kPi * m / n;
        t[m] = {float(std::cos(a)), float(-std::sin(a))};
    }
    return t;
}

template <int H, bool CONJ, int NZ>
void run_col(float2* ws, const float2* spec, const float2* tw, int h, int W2, int rows, int cap) {
    using C = zf::ColCfg<H>;
    int grid = (W2 + 1 + C::FPB - 1) / C::FPB;
    if (grid > cap) grid = cap;
    emu_launch(grid, C::THREADS, C::SMEM, zf::k_col_fused<H, CONJ, NZ>, ws, spec, tw, h, W2, rows);
}
template <int W2, int NZ>
void run_r2c(const float* tm, float2* ws, const float2* tw, int h, int w, int H, float sc, int cap) {
    using C = zf::RowCfg<W2>;
    int grid = (h + C::RPB - 1) / C::RPB;
    if (grid > cap) grid = cap;
    emu_launch(grid, C::THREADS, C::SMEM, zf::k_row_r2c<W2, NZ>, tm, ws, tw, h, w, H, sc);
}
template <int W2>
void run_c2r(const float2* ws, float* out, const float2* tw, int H, int orows, int ocols, int cap) {
    using C = zf::RowCfg<W2>;
    int grid = (orows + C::RPB - 1) / C::RPB;
    if (grid > cap) grid = cap;
    emu_launch(grid, C::THREADS, C::SMEM, zf::k_row_c2r<W2>, ws, out, tw, H, orows, ocols, ocols);
}

#define EMU_SIZES(X) X(64) X(128) X(256) X(120) X(240)

static void col(int H, bool conj, int nz, float2* ws, const float2* spec, const float2* tw, int h,
                int W2, int rows, int cap) {
#define X(N)                                                                                 \
    if (H == N) {                                                                            \
        if (conj) {                                                                          \
            if (nz == 1) return run_col<N, true, 1>(ws, spec, tw, h, W2, rows, cap);        \
            if (nz == 2) return run_col<N, true, 2>(ws, spec, tw, h, W2, rows, cap);        \
            return run_col<N, true, 0>(ws, spec, tw, h, W2, rows, cap);                     \
        }                                                                                    \
        if (nz == 1) return run_col<N, false, 1>(ws, spec, tw, h, W2, rows, cap);           \
        if (nz == 2) return run_col<N, false, 2>(ws, spec, tw, h, W2, rows, cap);           \
        return run_col<N, false, 0>(ws, spec, tw, h, W2, rows, cap);                        \
    }
    EMU_SIZES(X)
#undef X
    std::fprintf(stderr, "unsupported H %d\n", H);
    std::exit(2);
}
static void r2c(int W, int nz, const float* tm, float2* ws, const float2* tw, int h, int w, int H,
                float sc, int cap) {
#define X(N)                                                              \
    if (W == N) {                                                         \
        if (nz == 1) return run_r2c<N / 2, 1>(tm, ws, tw, h, w, H, sc, cap); \
        if (nz == 2) return run_r2c<N / 2, 2>(tm, ws, tw, h, w, H, sc, cap); \
        return run_r2c<N / 2, 0>(tm, ws, tw, h, w, H, sc, cap);              \
    }
    EMU_SIZES(X)
#undef X
    std::fprintf(stderr, "unsupported W %d\n", W);
    std::exit(2);
}
static void c2r(int W, const float2* ws, float* out, const float2* tw, int H, int orows, int ocols,
                int cap) {
#define X(N) \
    if (W == N) return run_c2r<N / 2>(ws, out, tw, H, orows, ocols, cap);
    EMU_SIZES(X)
#undef X
    std::fprintf(stderr, "unsupported W %d\n", W);
    std::exit(2);
}

int main(int argc, char** argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: zf_emu in.bin out.bin\n");
        return 2;
    }
    FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 2;
    int hd[11];
    if (std::fread(hd, sizeof(int), 11, f) != 11) return 2;
    const int B = hd[0], sy = hd[1], sx = hd[2], H = hd[3], W = hd[4], oy = hd[5], ox = hd[6];
    const bool conj = hd[7] != 0;
    const int cap = hd[8], nz_col = hd[9], nz_row = hd[10];
    const int W2 = W / 2;
    std::vector<float> tm((size_t)B * sy * sx);
    std::vector<float2> spec((size_t)(W2 + 1) * H);
    if (std::fread(tm.data(), sizeof(float), tm.size(), f) != tm.size()) return 2;
    if (std::fread(spec.data(), sizeof(float2), spec.size(), f) != spec.size()) return 2;
    std::fclose(f);

    // Exactly the workspace the library asks for: H * W/2 complex values.
    std::vector<float2> ws((size_t)H * W2);
    std::vector<float> out((size_t)B * oy * ox);
    auto twH = twiddles(H), twW = twiddles(W);
    const float scale = float(1.0 / (double(H) * double(W)));
    for (int t = 0; t < B; ++t) {
        r2c(W, nz_row, tm.data() + (size_t)t * sy * sx, ws.data(), twW.data(), sy, sx, H, scale, cap);
        col(H, conj, nz_col, ws.data(), spec.data(), twH.data(), sy, W2, oy, cap);
        c2r(W, ws.data(), out.data() + (size_t)t * oy * ox, twW.data(), H, oy, ox, cap);
    }
    FILE* g = std::fopen(argv[2], "wb");
    if (!g) return 2;
    std::fwrite(out.data(), sizeof(float), out.size(), g);
    std::fclose(g);
    return 0;
}
