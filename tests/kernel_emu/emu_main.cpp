// CPU execution of the library's CUDA kernels, for tests only.
//
// Each kernel block runs as blockDim std::threads sharing one shared-memory
// array and a std::barrier for __syncthreads; blocks run one after another.
// Built with AddressSanitizer, this checks the kernels' index arithmetic
// (every global and shared access in bounds) and their arithmetic against the
// oracle on small sizes before any of it runs on a GPU; it also checks that
// no barrier is divergent within a warp, that no bulk store's shared-memory
// source is written before the store's read is waited for, and (in the
// deferred-arrival mode) that no TMA-loaded buffer is read before its barrier
// wait.  It is never part of the library: the library has no CPU path.
//
// Usage: zf_emu <in.bin> <out.bin>, or zf_emu spectrum <in.bin> <out.bin>
//   in.bin : int32 header {B, sy, sx, H, W, oy, ox, conj, grid_cap, nz_col,
//            nz_row, chunk, max_mode, group (+ 1 << 16: workspace filled with
//            NaN first; + 1 << 17: TMA loads delivered only when a thread
//            polls their barrier)}, float32 templates [B][sy][sx],
//            complex64 spectrum [W/2+1][H]
//   out.bin: float32 [B][oy][ox] maps, or with max_mode the float32 [oy][ox]
//            running maximum and int32 [oy][ox] argmax over the templates,
//            followed with max_mode 2 by the float32 [oy][ox] sum and sum of
//            squares; max_mode 3: the maps followed by float32 [B] peaks
// spectrum mode (zfft_image_spectrum's two launches):
//   in.bin : int32 header {H, W, grid_cap (+ 1 << 17: TMA loads delivered
//            only when a thread polls their barrier)}, float32 image [H][W]
//   out.bin: complex64 [W/2+1][H]
#include <atomic>
#include <barrier>
#include <cmath>
#include <algorithm>
#include <map>
#include <memory>
#define INFINITY __builtin_inff()
#include <mutex>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <math.h>
#include <thread>
#include <vector>

// 8-byte aligned like CUDA's float2, so that the alignment sanitizer flags
// an 8-byte access at a 4-byte aligned address.
struct __attribute__((aligned(8))) float2 {
    float x, y;
};
struct __attribute__((aligned(8))) int2 {
    int x, y;
};
inline int2 make_int2(int x, int y) { return int2{x, y}; }
struct __attribute__((aligned(16))) float4 {
    float x, y, z, w;
};
struct dim3 {
    unsigned x = 1, y = 1, z = 1;
};
#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __launch_bounds__(...)
#define __grid_constant__

thread_local dim3 threadIdx, blockIdx, blockDim, gridDim;
thread_local std::barrier<>* emu_barrier = nullptr;
thread_local float2* emu_smem = nullptr;
thread_local size_t emu_smem_bytes = 0;
thread_local unsigned emu_or_calls = 0;
std::atomic<int> emu_or_flags[2];

// __syncthreads compiles to an .aligned barrier: every thread of a warp must
// execute the same barrier instruction.  Each arrival records its call site
// (the return address, distinct per template instantiation and call site);
// after the barrier every thread checks its warp-mates arrived from the same
// site, so barriers inside divergent branches abort the run.
thread_local unsigned emu_bar_calls = 0;
thread_local std::vector<void*>* emu_sites = nullptr;  // [2][blockDim]

static void emu_check_site(unsigned slot, void* site) {
    const unsigned n = blockDim.x;
    const unsigned w0 = threadIdx.x & ~31u;
    for (unsigned l = w0; l < w0 + 32 && l < n; ++l) {
        if (emu_sites[slot][l] != site) {
            std::fprintf(stderr, "divergent barrier: thread %u and %u of warp %u at different "
                                 "barrier instructions\n", threadIdx.x, l, w0 / 32);
            std::abort();
        }
    }
}
__attribute__((noinline)) void __syncthreads() {
    void* site = __builtin_return_address(0);
    const unsigned slot = emu_bar_calls++ & 1u;
    emu_sites[slot][threadIdx.x] = site;
    emu_barrier->arrive_and_wait();
    emu_check_site(slot, site);
}
__attribute__((noinline)) int __syncthreads_or(int pred) {
    void* site = __builtin_return_address(0);
    const unsigned slot = emu_bar_calls++ & 1u;
    emu_sites[slot][threadIdx.x] = site;
    const unsigned oslot = emu_or_calls++ & 1u;
    if (pred) emu_or_flags[oslot].store(1);
    emu_barrier->arrive_and_wait();
    emu_check_site(slot, site);
    const int r = emu_or_flags[oslot].load();
    emu_barrier->arrive_and_wait();  // plain barrier: everyone has read the flag
    if (threadIdx.x == 0) emu_or_flags[oslot].store(0);
    return r;
}
inline int atomicExch(int* p, int v) { return __atomic_exchange_n(p, v, __ATOMIC_SEQ_CST); }
inline unsigned atomicMax(unsigned* p, unsigned v) {
    unsigned cur = __atomic_load_n(p, __ATOMIC_SEQ_CST);
    while (cur < v && !__atomic_compare_exchange_n(p, &cur, v, false, __ATOMIC_SEQ_CST,
                                                   __ATOMIC_SEQ_CST)) {
    }
    return cur;
}
// Warp shuffles: every lane of the warp must call (full mask); each warp has
// an exchange array and a barrier of its lanes.
thread_local std::barrier<>* emu_warp_bar = nullptr;
thread_local float* emu_warp_buf = nullptr;
inline float __shfl_xor_sync(unsigned mask, float v, int lane_mask) {
    if (mask != 0xffffffffu) std::abort();
    const unsigned lane = threadIdx.x & 31u;
    emu_warp_buf[lane] = v;
    emu_warp_bar->arrive_and_wait();
    const float r = emu_warp_buf[lane ^ (unsigned)lane_mask];
    emu_warp_bar->arrive_and_wait();
    return r;
}
template <class T>
inline T __ldg(const T* p) {
    return *p;
}

#include "../../zipfft_b200/csrc/xcorr_kernels.cuh"

float2* zf::dyn_smem() { return emu_smem; }


// mbarrier stand-in: phase parity, pending arrivals, transaction bytes.
struct EmuBar {
    uint32_t phase = 0, count = 0, pending = 0;
    long long tx = 0;
};
static std::mutex emu_bar_mu;
static std::map<uint64_t*, EmuBar> emu_bars;
static void emu_bar_complete(EmuBar& b) {
    if (b.pending == 0 && b.tx == 0) {
        b.phase ^= 1u;
        b.pending = b.count;
    }
}
void zf::emu_mbar_init(uint64_t* bar, uint32_t count) {
    std::lock_guard<std::mutex> l(emu_bar_mu);
    EmuBar b;
    b.count = b.pending = count;
    emu_bars[bar] = b;
}
void zf::emu_mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    std::lock_guard<std::mutex> l(emu_bar_mu);
    EmuBar& b = emu_bars.at(bar);
    b.tx += bytes;
    if (b.pending == 0) std::abort();
    b.pending -= 1;
    emu_bar_complete(b);
}
void zf::emu_mbar_complete_tx(uint64_t* bar, uint32_t bytes) {
    std::lock_guard<std::mutex> l(emu_bar_mu);
    EmuBar& b = emu_bars.at(bar);
    b.tx -= bytes;
    emu_bar_complete(b);
}
// TMA loads: delivered at issue (a refill that lands while the buffer is
// still being read then corrupts the results), or with emu_defer_loads only
// when a thread next polls the load's barrier (a read of a buffer before its
// barrier wait then sees the old contents).  In deferred mode a block must
// not exit with a load still undelivered.
static bool emu_defer_loads = false;
struct EmuPendingLoad {
    uint64_t* bar;
    void* dst;
    std::vector<unsigned char> bytes;
};
static std::vector<EmuPendingLoad> emu_pending_loads;  // guarded by emu_bar_mu
void zf::emu_tma_arrive(void* dst, const void* data, uint32_t bytes, uint64_t* bar) {
    if (!emu_defer_loads) {
        std::memcpy(dst, data, bytes);
        emu_mbar_complete_tx(bar, bytes);
        return;
    }
    const auto* d = static_cast<const unsigned char*>(data);
    std::lock_guard<std::mutex> l(emu_bar_mu);
    emu_pending_loads.push_back({bar, dst, std::vector<unsigned char>(d, d + bytes)});
}
bool zf::emu_mbar_try_wait(uint64_t* bar, uint32_t parity) {
    std::lock_guard<std::mutex> l(emu_bar_mu);
    EmuBar& b = emu_bars.at(bar);
    for (size_t i = 0; i < emu_pending_loads.size();) {
        EmuPendingLoad& p = emu_pending_loads[i];
        if (p.bar != bar) {
            ++i;
            continue;
        }
        std::memcpy(p.dst, p.bytes.data(), p.bytes.size());
        b.tx -= (long long)p.bytes.size();
        emu_bar_complete(b);
        emu_pending_loads.erase(emu_pending_loads.begin() + (long)i);
    }
    return b.phase != parity;  // the phase with that parity completed
}
static size_t emu_pending_load_count() {
    std::lock_guard<std::mutex> l(emu_bar_mu);
    return emu_pending_loads.size();
}
// Bulk L2 prefetch rule: 16-byte aligned address and size; the emulator
// also reads the range, so ASan flags a prefetch outside any allocation.
void zf::emu_check_prefetch(const void* p, uint32_t bytes) {
    if (reinterpret_cast<uintptr_t>(p) % 16 || bytes % 16 || bytes == 0) {
        std::fprintf(stderr, "bad L2 prefetch %p %u\n", p, bytes);
        std::abort();
    }
    volatile unsigned char sink = 0;
    const unsigned char* c = static_cast<const unsigned char*>(p);
    sink = sink + c[0] + c[bytes - 1];
    (void)sink;
}
// discard.global.L2 rule: whole 128-byte lines only.  The line's contents
// are undefined afterwards: the harness fills it with NaN, so that a line
// dropped before its last reader shows up in the results.
void zf::emu_discard_line(const void* p) {
    if (reinterpret_cast<uintptr_t>(p) % 128) {
        std::fprintf(stderr, "misaligned L2 discard %p\n", p);
        std::abort();
    }
    float* f = static_cast<float*>(const_cast<void*>(p));
    for (int i = 0; i < 32; ++i) f[i] = NAN;
}
// Bulk store rules: 16-byte aligned addresses and sizes, source inside the
// block's shared memory.
void zf::emu_check_store(const void* dst, const void* src, uint32_t bytes) {
    const auto d = reinterpret_cast<uintptr_t>(dst), s = reinterpret_cast<uintptr_t>(src);
    const auto lo = reinterpret_cast<uintptr_t>(emu_smem);
    if (d % 16 || s % 16 || bytes % 16 || s < lo || s + bytes > lo + emu_smem_bytes) {
        std::fprintf(stderr, "bad bulk store dst=%p src=%p bytes=%u\n", dst, src, bytes);
        std::abort();
    }
}
// Bulk stores in flight, per issuing thread: the source bytes as they were at
// issue.  The GPU may read the source at any time until the issuing thread's
// wait_group.read, so a write to it before that wait (by any thread, or by a
// TMA load refilling the buffer) races with the store; the wait checks that
// the source still holds the recorded bytes.  A block must wait for all its
// stores before it exits (checked after each block).
struct EmuPendingStore {
    const unsigned char* src;
    std::vector<unsigned char> bytes;
};
thread_local std::vector<EmuPendingStore> emu_pending_stores;
void zf::emu_store_issued(const void* src, uint32_t bytes) {
    const auto* s = static_cast<const unsigned char*>(src);
    emu_pending_stores.push_back({s, std::vector<unsigned char>(s, s + bytes)});
}
void zf::emu_store_wait_read() {
    for (const auto& p : emu_pending_stores) {
        if (std::memcmp(p.src, p.bytes.data(), p.bytes.size()) != 0) {
            std::fprintf(stderr, "bulk store source %p overwritten before the store's read "
                                 "was waited for (thread %u, block %u)\n",
                         static_cast<const void*>(p.src), threadIdx.x, blockIdx.x);
            std::abort();
        }
    }
    emu_pending_stores.clear();
}

// TMA rules: 16-byte aligned addresses and sizes, destination inside the
// block's shared memory.
void zf::emu_check_copy(const void* dst, const void* src, uint32_t bytes) {
    const auto d = reinterpret_cast<uintptr_t>(dst), s = reinterpret_cast<uintptr_t>(src);
    const auto lo = reinterpret_cast<uintptr_t>(emu_smem);
    if (d % 16 || s % 16 || bytes % 16 || d < lo || d + bytes > lo + emu_smem_bytes) {
        std::fprintf(stderr, "bad TMA copy dst=%p src=%p bytes=%u\n", dst, src, bytes);
        std::abort();
    }
}

template <class K, class... A>
void emu_launch(dim3 grid, int block, size_t smem_bytes, K kernel, A... args) {
    // 128-byte aligned like the device's dynamic shared memory.
    std::vector<float4> store((smem_bytes + 15) / 16 + 8);
    float2* smem = reinterpret_cast<float2*>((reinterpret_cast<uintptr_t>(store.data()) + 127) & ~uintptr_t(127));
    std::barrier<> bar(block);
    std::vector<void*> sites[2] = {std::vector<void*>(block), std::vector<void*>(block)};
    const int nwarps = (block + 31) / 32;
    std::vector<std::unique_ptr<std::barrier<>>> wbars;
    for (int w = 0; w < nwarps; ++w)
        wbars.push_back(std::make_unique<std::barrier<>>(std::min(32, block - 32 * w)));
    std::vector<float> wbuf((size_t)nwarps * 32);
    std::vector<std::thread> threads;
    for (int tid = 0; tid < block; ++tid) {
        threads.emplace_back([&, tid] {
            threadIdx.x = tid;
            blockDim.x = block;
            gridDim = grid;
            emu_barrier = &bar;
            emu_smem = smem;
            emu_smem_bytes = smem_bytes;
            emu_or_calls = 0;
            emu_bar_calls = 0;
            emu_sites = sites;
            emu_warp_bar = wbars[tid / 32].get();
            emu_warp_buf = wbuf.data() + (tid / 32) * 32;
            for (unsigned by = 0; by < grid.y; ++by) {
                for (unsigned bx = 0; bx < grid.x; ++bx) {
                    blockIdx.x = bx;
                    blockIdx.y = by;
                    kernel(args...);
                    if (!emu_pending_stores.empty()) {
                        std::fprintf(stderr, "block %u exited with %zu bulk store(s) not waited "
                                             "for (thread %d)\n",
                                     bx, emu_pending_stores.size(), tid);
                        std::abort();
                    }
                    bar.arrive_and_wait();
                    if (tid == 0 && emu_pending_load_count() != 0) {
                        std::fprintf(stderr, "block %u exited with %zu TMA load(s) in flight\n",
                                     bx, emu_pending_load_count());
                        std::abort();
                    }
                    bar.arrive_and_wait();  // the check precedes the next block's loads
                }
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

static int g_status = 0;

// Per-thread twiddle tables (Stockham::fill_thread_twiddles), built on the
// host from the same root table the kernels' loads would read, as the
// library builds them on the device.
template <class P, int TN>
static std::vector<float4> thread_twiddles(const float2* roots) {
    std::vector<float4> tab((size_t)P::TWU * P::kThreads);
    for (int t = 0; t < P::kThreads; ++t) P::template fill_thread_twiddles<TN>(tab.data(), roots, t);
    return tab;
}
template <int N>
using RowPlanOf = zf::Stockham<N / 2, zf::fft_threads(N / 2), false, false>;
template <int N>
using ColPlanOf = zf::Stockham<N, zf::fft_threads(N), false, false>;
template <int N>
using RevPlanOf = zf::Stockham<N, zf::fft_threads(N), true, true>;

template <int H, bool CONJ, int NZ>
void run_col(float2* Q, const float2* R, int r_pitch, const float2* spec, const float2* tw, int h,
             int W2, int rows, int nt, long long qts, long long rts, int cap) {
    using C = zf::ColCfg<H, NZ>;
    int grid = (W2 + C::FPB) / C::FPB * nt;
    if (grid > cap) grid = cap;
    const auto tt = thread_twiddles<ColPlanOf<H>, H>(tw);
    const auto tr = thread_twiddles<RevPlanOf<H>, H>(tw);
    emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, C::SMEM, zf::k_col_fused<H, CONJ, NZ>, Q, R,
               r_pitch, spec, tt.data(), tr.data(), h, W2, rows, R != Q ? 1 : 0, nt, qts, rts,
               &g_status);
}
template <int W2, int NZ>
void run_r2c(const float* tm, float2* R, const float2* tw, int h, int w, int r_pitch,
             long long r_tstride, int nt, float sc, int cap) {
    using C = zf::R2cCfg<W2>;
    int units = ((h + 1) / 2 * 2 + C::RPB - 1) / C::RPB * nt;
    int grid = units < cap ? units : cap;
    const auto tt = thread_twiddles<RowPlanOf<2 * W2>, 2 * W2>(tw);
    emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, C::SMEM, zf::k_row_r2c<W2, NZ>, tm, R, tw,
               tt.data(), h, w, r_pitch, r_tstride, nt, sc);
}
template <int H>
void run_col_fwd(float2* spec, const float2* tw, int W2, int cap) {
    using C = zf::ColFwdCfg<H>;
    int grid = (W2 + C::FPB - 1) / C::FPB;
    if (grid > cap) grid = cap;
    const auto tt = thread_twiddles<ColPlanOf<H>, H>(tw);
    emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, C::SMEM, zf::k_col_fwd<H>, spec, tt.data(),
               W2, &g_status);
}
template <int W2>
void run_c2r(const float2* Q, int H, float* out, int* arg, float* sum, float* sumsq,
             unsigned* peak, const float2* tw, int orows, int ocols, int tindex, int reset,
             int nt, long long ots, int cap) {
    using C = zf::C2rCfg<W2>;
    zf::CUtensorMap map{reinterpret_cast<const unsigned char*>(Q), H, W2 * nt, (long long)H * 8,
                        C::RPB, C::BOXK, 8};
    // As the library's launcher: the running-map modes give each block whole
    // row groups (all nt templates of each), the map modes (template, group)
    // units.
    int groups = (orows + C::RPB - 1) / C::RPB * (arg ? 1 : nt);
    const auto ttr = thread_twiddles<RowPlanOf<2 * W2>, 2 * W2>(tw);
    const auto ttc = thread_twiddles<ColPlanOf<2 * W2>, 2 * W2>(tw);
    int grid = groups < cap ? groups : cap;
    float* nf = nullptr;
    unsigned* np = nullptr;
    if (arg && sum)
        emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, C::SMEM,
                   zf::k_row_c2r<W2, zf::kRunningStats>, map, out, arg, sum, sumsq, np, tw, ttr.data(), orows,
                   ocols, ocols, tindex, reset, nt, ots, &g_status);
    else if (arg && sumsq)
        emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, C::SMEM,
                   zf::k_row_c2r<W2, zf::kRunningSumSq>, map, out, arg, nf, sumsq, np, tw, ttr.data(), orows,
                   ocols, ocols, tindex, reset, nt, ots, &g_status);
    else if (arg)
        emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, C::SMEM, zf::k_row_c2r<W2, zf::kRunningMax>,
                   map, out, arg, nf, nf, np, tw, ttr.data(), orows, ocols, ocols, tindex, reset, nt, ots,
                   &g_status);
    else if (ocols == 2 * W2 && reinterpret_cast<uintptr_t>(out) % 8 == 0 && ots % 2 == 0) {
        // full aligned maps: the W/2-point form, as the library launches it
        if (peak)
            emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, C::SMEM,
                       zf::k_row_c2r<W2, zf::kStorePeak>, map, out, (int*)nullptr, nf, nf, peak, tw, ttr.data(),
                       orows, ocols, ocols, 0, 0, nt, ots, &g_status);
        else
            emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, C::SMEM,
                       zf::k_row_c2r<W2, zf::kStoreMap>, map, out, (int*)nullptr, nf, nf, np, tw, ttr.data(),
                       orows, ocols, ocols, 0, 0, nt, ots, &g_status);
    } else if (peak)  // cropped maps: the row-pair form
        emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, zf::C2rPairCfg<W2>::SMEM,
                   zf::k_row_c2r_pair<W2, zf::kStorePeak>, map, out, peak, ttc.data(), orows, ocols, ocols,
                   nt, ots, &g_status);
    else
        emu_launch(dim3{(unsigned)grid, 1, 1}, C::THREADS, zf::C2rPairCfg<W2>::SMEM,
                   zf::k_row_c2r_pair<W2, zf::kStoreMap>, map, out, np, ttc.data(), orows, ocols, ocols, nt,
                   ots, &g_status);
}

#define EMU_SIZES(X) X(64) X(128) X(256) X(512) X(2048) X(120) X(240)

static void col(int H, bool conj, int nz, float2* Q, const float2* R, int rp, const float2* spec,
                const float2* tw, int h, int W2, int rows, int cap, int nt = 1, long long qts = 0,
                long long rts = 0) {
#define X(N)                                                                                   \
    if (H == N) {                                                                              \
        if (conj) {                                                                            \
            if (nz == 1) return run_col<N, true, 1>(Q, R, rp, spec, tw, h, W2, rows, nt, qts, rts, cap); \
            if (nz == 2) return run_col<N, true, 2>(Q, R, rp, spec, tw, h, W2, rows, nt, qts, rts, cap); \
            return run_col<N, true, 0>(Q, R, rp, spec, tw, h, W2, rows, nt, qts, rts, cap);  \
        }                                                                                      \
        if (nz == 1) return run_col<N, false, 1>(Q, R, rp, spec, tw, h, W2, rows, nt, qts, rts, cap); \
        if (nz == 2) return run_col<N, false, 2>(Q, R, rp, spec, tw, h, W2, rows, nt, qts, rts, cap); \
        return run_col<N, false, 0>(Q, R, rp, spec, tw, h, W2, rows, nt, qts, rts, cap);     \
    }
    EMU_SIZES(X)
#undef X
    std::fprintf(stderr, "unsupported H %d\n", H);
    std::exit(2);
}
static void r2c(int W, int nz, const float* tm, float2* R, const float2* tw, int h, int w, int rp,
                long long rts, int nt, float sc, int cap) {
#define X(N)                                                                           \
    if (W == N) {                                                                      \
        if (nz == 1) return run_r2c<N / 2, 1>(tm, R, tw, h, w, rp, rts, nt, sc, cap);  \
        if (nz == 2) return run_r2c<N / 2, 2>(tm, R, tw, h, w, rp, rts, nt, sc, cap);  \
        return run_r2c<N / 2, 0>(tm, R, tw, h, w, rp, rts, nt, sc, cap);               \
    }
    EMU_SIZES(X)
#undef X
    std::fprintf(stderr, "unsupported W %d\n", W);
    std::exit(2);
}
static void c2r(int W, const float2* Q, int H, float* out, int* arg, float* sum, float* sumsq,
                unsigned* peak, const float2* tw, int orows, int ocols, int tindex, int reset,
                int cap, int nt = 1, long long ots = 0) {
#define X(N)                                                                                    \
    if (W == N)                                                                                 \
        return run_c2r<N / 2>(Q, H, out, arg, sum, sumsq, peak, tw, orows, ocols, tindex, reset, \
                              nt, ots, cap);
    EMU_SIZES(X)
#undef X
    std::fprintf(stderr, "unsupported W %d\n", W);
    std::exit(2);
}

static void col_fwd(int H, float2* spec, const float2* tw, int W2, int cap) {
#define X(N) \
    if (H == N) return run_col_fwd<N>(spec, tw, W2, cap);
    EMU_SIZES(X)
#undef X
    std::fprintf(stderr, "unsupported H %d\n", H);
    std::exit(2);
}

// The host sequence of zfft_image_spectrum: the unscaled row pass over all
// image rows into the output (pitch H), then the in-place column pass.
static int spectrum_main(const char* in, const char* outp) {
    FILE* f = std::fopen(in, "rb");
    if (!f) return 2;
    int hd[3];
    if (std::fread(hd, sizeof(int), 3, f) != 3) return 2;
    const int H = hd[0], W = hd[1], cap = hd[2] & 0xFFFF;
    emu_defer_loads = (hd[2] >> 17) & 1;  // TMA loads land at the wait
    std::vector<float> img((size_t)H * W);
    if (std::fread(img.data(), sizeof(float), img.size(), f) != img.size()) return 2;
    std::fclose(f);
    const size_t n = (size_t)(W / 2 + 1) * H;
    std::vector<float4> store(n / 2 + 1);
    float2* spec = reinterpret_cast<float2*>(store.data());
    auto twH = twiddles(H), twW = twiddles(W);
    r2c(W, 0, img.data(), spec, twW.data(), H, W, H, 0, 1, 1.0f, cap);
    col_fwd(H, spec, twH.data(), W / 2, cap);
    if (g_status != 0) {
        std::fprintf(stderr, "device status %d\n", g_status);
        return 3;
    }
    FILE* g = std::fopen(outp, "wb");
    if (!g) return 2;
    std::fwrite(spec, sizeof(float2), n, g);
    std::fclose(g);
    return 0;
}

int main(int argc, char** argv) {
    if (argc == 4 && std::strcmp(argv[1], "spectrum") == 0) return spectrum_main(argv[2], argv[3]);
    if (argc != 3) {
        std::fprintf(stderr, "usage: zf_emu in.bin out.bin\n");
        return 2;
    }
    FILE* f = std::fopen(argv[1], "rb");
    if (!f) return 2;
    int hd[14];
    if (std::fread(hd, sizeof(int), 14, f) != 14) return 2;
    const int B = hd[0], sy = hd[1], sx = hd[2], H = hd[3], W = hd[4], oy = hd[5], ox = hd[6];
    const bool conj = hd[7] != 0;
    const int cap = hd[8], nz_col = hd[9], nz_row = hd[10], chunk = hd[11];
    const bool max_mode = hd[12] == 1 || hd[12] == 2 || hd[12] == 4;  // running max / argmax maps
    const bool stats = hd[12] == 2 || hd[12] == 4;  // ... and sum (not with 4) / sum-of-squares maps
    const bool no_sum = hd[12] == 4;                // the sum of squares alone (sum stays 0)
    const bool peaks_mode = hd[12] == 3;               // maps plus per-template peaks
    const int group = hd[13] & 0xFFFF;                   // >= 2: batched groups
    const bool poison = (hd[13] >> 16) & 1;              // workspace starts as NaN
    emu_defer_loads = (hd[13] >> 17) & 1;                // TMA loads land at the wait
    // max_mode 2 with bit 18: every second template starts a new "batch"
    // whose first template overwrites only the sum maps (reset kResetSums),
    // as the search's per-batch partial sums do; the maximum keeps running.
    // With batched groups, every group after the first starts a new batch.
    const bool sum_batches = (hd[13] >> 18) & 1;
    const int W2 = W / 2;
    std::vector<float> tm((size_t)B * sy * sx);
    std::vector<float2> spec((size_t)(W2 + 1) * H);
    if (std::fread(tm.data(), sizeof(float), tm.size(), f) != tm.size()) return 2;
    if (std::fread(spec.data(), sizeof(float2), spec.size(), f) != spec.size()) return 2;
    std::fclose(f);

    // The host orchestration of zfft_padded_real_{corr,conv}_2d: Q (H x W2)
    // first; with chunk > 0 the rows of `chunk` templates go to a region
    // after Q with pitch round_up(h, 2), else into rows [0, h) of Q.
    const long long h_pad = (sy + 1) / 2 * 2;
    const long long q_elems = (long long)H * W2, r_elems = (long long)W2 * h_pad;
    const long long ws_elems = group >= 2 ? group * q_elems
                                          : q_elems + (chunk > 0 ? chunk : 0) * r_elems;
    std::vector<float4> ws_store((ws_elems + 1) / 2 + 1);
    float2* Q = reinterpret_cast<float2*>(ws_store.data());
    if (poison)
        for (auto& v4 : ws_store) v4 = float4{NAN, NAN, NAN, NAN};
    float2* Rregion = Q + q_elems;
    std::vector<float> out((size_t)(max_mode ? 1 : B) * oy * ox);
    std::vector<int> arg(max_mode ? (size_t)oy * ox : 0);
    std::vector<float> sum(stats ? (size_t)oy * ox : 0), sumsq(stats ? (size_t)oy * ox : 0);
    float* sum_p = stats && !no_sum ? sum.data() : nullptr;
    float* sumsq_p = stats ? sumsq.data() : nullptr;
    std::vector<unsigned> peak_keys(peaks_mode ? B : 0, 0u);
    auto twH = twiddles(H), twW = twiddles(W);
    const float scale = float(1.0 / (double(H) * double(W)));
    // Batched groups: each template of a group in its own Q slice, rows
    // first in rows [0, h) of the slice, one launch per kernel per group.
    for (int t0 = 0; group >= 2 && t0 < B; t0 += group) {
        const int n = B - t0 < group ? B - t0 : group;
        r2c(W, nz_row, tm.data() + (size_t)t0 * sy * sx, Q, twW.data(), sy, sx, H, q_elems, n,
            scale, cap);
        col(H, conj, nz_col, Q, Q, H, spec.data(), twH.data(), sy, W2, oy, cap, n, q_elems,
            q_elems);
        // the tile map spans the whole group's slices, as on the device
        if (max_mode)  // the group's templates folded into the running maps
            c2r(W, Q, H, out.data(), arg.data(), sum_p, sumsq_p, nullptr, twW.data(), oy, ox, t0,
                t0 == 0 ? zf::kResetMax : (sum_batches ? zf::kResetSums : 0), cap, n, 0);
        else
            c2r(W, Q, H, out.data() + (size_t)t0 * oy * ox, nullptr, nullptr, nullptr,
                peaks_mode ? peak_keys.data() + t0 : nullptr, twW.data(), oy, ox, 0, 0, cap, n,
                (long long)oy * ox);
    }
    const int step = chunk > 0 ? chunk : 1;
    for (int t0 = 0; group < 2 && t0 < B; t0 += step) {
        const int n = B - t0 < step ? B - t0 : step;
        if (chunk > 0)
            r2c(W, nz_row, tm.data() + (size_t)t0 * sy * sx, Rregion, twW.data(), sy, sx, (int)h_pad,
                r_elems, n, scale, cap);
        for (int j = 0; j < n; ++j) {
            const int t = t0 + j;
            const float2* Rt = Q;
            int rp = H;
            if (chunk > 0) {
                Rt = Rregion + (size_t)j * r_elems;
                rp = (int)h_pad;
            } else {
                r2c(W, nz_row, tm.data() + (size_t)t * sy * sx, Q, twW.data(), sy, sx, H, 0, 1, scale, cap);
            }
            col(H, conj, nz_col, Q, Rt, rp, spec.data(), twH.data(), sy, W2, oy, cap);
            if (max_mode)
                c2r(W, Q, H, out.data(), arg.data(), sum_p, sumsq_p, nullptr, twW.data(), oy, ox, t,
                    t == 0 ? zf::kResetMax : ((sum_batches && t % 2 == 0) ? zf::kResetSums : 0),
                    cap);
            else
                c2r(W, Q, H, out.data() + (size_t)t * oy * ox, nullptr, nullptr, nullptr,
                    peaks_mode ? peak_keys.data() + t : nullptr, twW.data(), oy, ox, 0, 0, cap);
        }
    }
    if (g_status != 0) {
        std::fprintf(stderr, "device status %d\n", g_status);
        return 3;
    }
    FILE* g = std::fopen(argv[2], "wb");
    if (!g) return 2;
    std::fwrite(out.data(), sizeof(float), out.size(), g);
    if (max_mode) std::fwrite(arg.data(), sizeof(int), arg.size(), g);
    if (stats) {
        std::fwrite(sum.data(), sizeof(float), sum.size(), g);
        std::fwrite(sumsq.data(), sizeof(float), sumsq.size(), g);
    }
    for (unsigned k : peak_keys) {
        const float v = zf::key_value(k);
        std::fwrite(&v, sizeof(float), 1, g);
    }
    std::fclose(g);
    return 0;
}
