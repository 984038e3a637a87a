// extern "C" entry points of libzipfft_b200.so (declared in include/zipfft_b200.h).
//
// Mirrors the validation and dispatch of zipFFT's binding
// (src/cuda/real_conv_2d_binding.cu:189-285) and launcher
// (src/cuda/real_conv_2d.cuh:153-293) with these differences:
//   * shapes are run-time values (only the FFT sizes are compiled in);
//   * errors are returned as status codes with a message, never std::exit
//     (zipfft_common.hpp:20-41) and never silently ignored (binding.cu:284);
//   * the output may be the valid crop (as the reference) or the full map;
//   * the per-call cudaFuncSetAttribute / workspace creation of the reference
//     (cuh:243-259) happen once per device.
#include <cmath>
#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/zipfft_b200.h"
#include "async_copy.cuh"
#include "fft_core.cuh"
#include "launch.h"

namespace zf {
__global__ void k_peak_values(unsigned* keys, int n);
}

namespace {

constexpr int kVersion = 300;  // 0.3.0
constexpr int kMaxDevices = 64;
constexpr int kMaxChunk = 32;  // templates per row-r2c launch, and per batched group

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

// ZFFT_TRACE=1: print every step of a call to stderr and synchronize after
// each kernel launch (debugging aid, like CUDA_LAUNCH_BLOCKING).
bool trace_on() {
    static const bool on = [] {
        const char* v = std::getenv("ZFFT_TRACE");
        return v && v[0] && v[0] != '0';
    }();
    return on;
}
void trace(const char* fmt, ...) {
    if (!trace_on()) return;
    va_list ap;
    va_start(ap, fmt);
    std::fprintf(stderr, "[zfft] ");
    std::vfprintf(stderr, fmt, ap);
    std::fprintf(stderr, "\n");
    std::fflush(stderr);
    va_end(ap);
}
cudaError_t trace_sync(cudaStream_t s, const char* what, int t) {
    if (!trace_on()) return cudaSuccess;
    trace("launched %s (template %d); synchronizing", what, t);
    cudaError_t e = cudaStreamSynchronize(s);
    trace("%s (template %d) done: %s", what, t, cudaGetErrorString(e));
    return e;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(ZFFT_ERROR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// ---------------------------------------------------------------------------
// Twiddle tables: w_N[m] = exp(-2 pi i m / N), one table per supported size,
// computed in double precision on the host and uploaded once per device.
// ---------------------------------------------------------------------------
__device__ __align__(16) float2 g_tw_pool[ZF_TW_POOL_TOTAL];

// Device status word: kernels that give up on a bounded wait write a
// ZFFT_ERROR_* code here; zfft_check_device_status reads and clears it.
__device__ int g_status;
// 16-byte source of the bounded-wait self-test copy.
__device__ __align__(16) float4 g_selftest_src;

int tw_offset(int n) {
    int off = 0;
#define ZF_X(N)              \
    if (n == (N)) return off; \
    off += (N);
    ZF_FOR_EACH_FFT_SIZE(ZF_X)
#undef ZF_X
    return -1;
}

// Scratch of zfft_padded_real_corr_2d_noalloc: a fixed 16 MiB array in the
// library's own device memory (one per GPU that loads the library, held until
// the process exits), so that entry point never allocates.  Host code must
// not use g_noalloc_ws as a pointer: it is a host-side stand-in for the
// symbol; the device address comes from cudaGetSymbolAddress.
constexpr size_t kNoAllocBytes = size_t(16) << 20;
__device__ __align__(256) float2 g_noalloc_ws[kNoAllocBytes / sizeof(float2)];

// The number of visible devices, read once: it cannot change while the
// process runs, and the calls validate their device index against it.
cudaError_t device_count(int* n) {
    static std::atomic<int> cached{-1};
    int c = cached.load(std::memory_order_relaxed);
    if (c < 0) {
        cudaError_t e = cudaGetDeviceCount(&c);
        if (e != cudaSuccess) return e;
        cached.store(c, std::memory_order_relaxed);
    }
    *n = c;
    return cudaSuccess;
}

std::mutex g_init_mu;
bool g_dev_ready[kMaxDevices];
float2* g_dev_pool[kMaxDevices];
int* g_dev_status[kMaxDevices];

int ensure_device(int device) {
    std::lock_guard<std::mutex> lock(g_init_mu);
    if (g_dev_ready[device]) return ZFFT_SUCCESS;
    std::vector<float2> host(ZF_TW_POOL_TOTAL);
#define ZF_X(N)                                                      \
    {                                                                \
        const int o = tw_offset(N);                                  \
        for (int m = 0; m < (N); ++m) {                              \
            const double a = 2.0 * zf::kPi * double(m) / double(N);  \
            host[o + m].x = float(std::cos(a));                      \
            host[o + m].y = float(-std::sin(a));                     \
        }                                                            \
    }
    ZF_FOR_EACH_FFT_SIZE(ZF_X)
#undef ZF_X
    cudaError_t e = cudaMemcpyToSymbol(g_tw_pool, host.data(), sizeof(float2) * host.size());
    if (e != cudaSuccess) return cuda_fail(e, "uploading twiddle tables");
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_tw_pool);
    if (e != cudaSuccess) return cuda_fail(e, "resolving twiddle table address");
    g_dev_pool[device] = static_cast<float2*>(p);
    e = cudaGetSymbolAddress(&p, g_status);
    if (e != cudaSuccess) return cuda_fail(e, "resolving device status address");
    g_dev_status[device] = static_cast<int*>(p);
    // Per-thread twiddle tables of every size's kernels, built on the device
    // from the root tables (once; this first call synchronizes the device).
#define ZF_X(N)                                                                   \
    if ((e = zf::init_thread_twiddles_##N(g_dev_pool[device] + tw_offset(N), device)) != \
        cudaSuccess)                                                              \
        return cuda_fail(e, "building the per-thread twiddle tables");
    ZF_FOR_EACH_FFT_SIZE(ZF_X)
#undef ZF_X
    if ((e = cudaDeviceSynchronize()) != cudaSuccess)
        return cuda_fail(e, "building the per-thread twiddle tables");
    g_dev_ready[device] = true;
    return ZFFT_SUCCESS;
}

// RAII: make `device` current for the call, restore the caller's device.
struct DeviceGuard {
    int prev = -1;
    cudaError_t err = cudaSuccess;
    explicit DeviceGuard(int device) {
        err = cudaGetDevice(&prev);
        if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

bool supported(int n) { return tw_offset(n) >= 0; }

// ---------------------------------------------------------------------------
// Opt-in per-stage timing for benchmarks: while enabled on the calling thread,
// events are recorded on the call's stream around every kernel launch, and
// zfft_stage_timing_read sums their intervals per stage.
// ---------------------------------------------------------------------------
constexpr int kStages = 3;  // 0: row r2c, 1: column, 2: row c2r
struct StageTimer {
    bool on = false;
    int device = -1;
    std::vector<cudaEvent_t> pool;      // reusable events
    std::vector<std::pair<int, int>> marks[kStages];  // (start, stop) indices into pool
    size_t used = 0;
    cudaEvent_t next(cudaError_t* e) {
        if (used == pool.size()) {
            cudaEvent_t ev;
            *e = cudaEventCreate(&ev);
            if (*e != cudaSuccess) return nullptr;
            pool.push_back(ev);
        }
        return pool[used++];
    }
};
thread_local StageTimer g_timer;

// Record the start of a stage launch; returns the pool index (or -1).
int timer_mark(cudaStream_t s) {
    if (!g_timer.on) return -1;
    cudaError_t e = cudaSuccess;
    cudaEvent_t ev = g_timer.next(&e);
    if (!ev || cudaEventRecord(ev, s) != cudaSuccess) return -1;
    return int(g_timer.used - 1);
}
void timer_close(int stage, int start, cudaStream_t s) {
    if (start < 0) return;
    int stop = timer_mark(s);
    if (stop >= 0) g_timer.marks[stage].push_back({start, stop});
}

using ColFn = cudaError_t (*)(float2*, const float2*, int, const float2*, const float2*, int, int,
                              int, bool, int, bool, int, long long, long long, int*, int,
                              cudaStream_t);
using R2cFn = cudaError_t (*)(const float*, float2*, const float2*, int, int, int, long long, int,
                              float, int, int, cudaStream_t);
using ColFwdFn = cudaError_t (*)(float2*, const float2*, int, int*, int, cudaStream_t);
using QmapFn = cudaError_t (*)(const float2*, int, int, CUtensorMap*);
using C2rFn = cudaError_t (*)(const CUtensorMap*, float*, int*, float*, float*, unsigned*,
                              const float2*, int, int, int, int, int, int, long long, int*, int,
                              cudaStream_t);

ColFn col_fn(int n) {
#define ZF_X(N) \
    if (n == (N)) return zf::launch_col_##N;
    ZF_FOR_EACH_FFT_SIZE(ZF_X)
#undef ZF_X
    return nullptr;
}
R2cFn r2c_fn(int n) {
#define ZF_X(N) \
    if (n == (N)) return zf::launch_row_r2c_##N;
    ZF_FOR_EACH_FFT_SIZE(ZF_X)
#undef ZF_X
    return nullptr;
}
ColFwdFn col_fwd_fn(int n) {
#define ZF_X(N) \
    if (n == (N)) return zf::launch_col_fwd_##N;
    ZF_FOR_EACH_FFT_SIZE(ZF_X)
#undef ZF_X
    return nullptr;
}
QmapFn qmap_fn(int n) {
#define ZF_X(N) \
    if (n == (N)) return zf::make_qmap_##N;
    ZF_FOR_EACH_FFT_SIZE(ZF_X)
#undef ZF_X
    return nullptr;
}
C2rFn c2r_fn(int n) {
#define ZF_X(N) \
    if (n == (N)) return zf::launch_row_c2r_##N;
    ZF_FOR_EACH_FFT_SIZE(ZF_X)
#undef ZF_X
    return nullptr;
}

// Number of possibly non-zero inputs per stage-0 butterfly of an n-point
// transform whose first `len` inputs are non-zero: 1, 2 or 0 (= more).
int stage0_nz(int n, int len) {
    const int nb0 = n / zf::plan_first_radix(n);
    const int nz = (len + nb0 - 1) / nb0;
    return nz <= 2 ? (nz < 1 ? 1 : nz) : 0;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// zipFFT's compile-time shape table (real_conv_2d_binding.cu:51-106) -- every
// entry runs here -- followed by the 2DTM shapes this library is measured on.
const int kConfigs[][6] = {
    {48, 48, 64, 64, 1, 0},       {48, 48, 64, 64, 8, 0},       {96, 96, 128, 128, 1, 0},
    {96, 96, 128, 128, 8, 0},     {192, 192, 256, 256, 1, 0},   {192, 192, 256, 256, 4, 0},
    {384, 384, 512, 512, 1, 0},   {384, 384, 512, 512, 4, 0},   {384, 192, 512, 256, 1, 0},
    {384, 192, 512, 256, 4, 0},   {192, 384, 256, 512, 1, 0},   {192, 384, 256, 512, 4, 0},
    {48, 48, 64, 64, 1, 1},       {48, 48, 64, 64, 8, 1},       {96, 96, 128, 128, 1, 1},
    {96, 96, 128, 128, 8, 1},     {192, 192, 256, 256, 1, 1},   {192, 192, 256, 256, 4, 1},
    {384, 384, 512, 512, 1, 1},   {384, 384, 512, 512, 4, 1},   {384, 192, 512, 256, 1, 1},
    {384, 192, 512, 256, 4, 1},   {192, 384, 256, 512, 1, 1},   {192, 384, 256, 512, 4, 1},
    {16, 16, 64, 64, 1, 1},       {16, 16, 64, 64, 8, 1},       {32, 32, 128, 128, 1, 1},
    {32, 32, 128, 128, 8, 1},     {64, 64, 256, 256, 1, 1},     {64, 64, 256, 256, 4, 1},
    {128, 128, 512, 512, 1, 1},   {128, 128, 512, 512, 4, 1},   {128, 64, 512, 256, 1, 1},
    {128, 64, 512, 256, 4, 1},    {64, 128, 256, 512, 1, 1},    {64, 128, 256, 512, 4, 1},
    {512, 512, 4096, 4096, 1, 1}, {512, 512, 4096, 4096, 4, 1}, {512, 512, 4096, 4096, 8, 1},
    {512, 512, 4096, 4096, 12, 1}, {512, 512, 4096, 4096, 16, 1}, {512, 512, 4096, 4096, 20, 1},
    {512, 512, 4096, 4096, 24, 1}, {512, 512, 4096, 4096, 28, 1}, {512, 512, 4096, 4096, 32, 1},
    // 2DTM workloads: 1024^2 / 128^2, 4096^2 / 256^2, 4096^2 / 512^2,
    // 3840^2 / 384^2 (radix-3/5 path), 4096^2 / 384^2.
    {128, 128, 1024, 1024, 4, 1}, {256, 256, 4096, 4096, 32, 1}, {512, 512, 4096, 4096, 64, 1},
    {384, 384, 3840, 3840, 128, 1}, {384, 384, 4096, 4096, 256, 1},
};

// One call of the correlation path.  arg == nullptr: output holds `batch`
// maps of oy x ox.  Otherwise output / arg are the running max / argmax maps
// (oy x ox) that every template folds into, template t with index
// tindex_base + t; reset (zf::kResetMax / kResetSums bits): the first
// template overwrites every map / only the sum maps.  With sum (and
// sumsq) also given, every template is added to those maps as well.  With
// peaks (maps mode only), peaks[t] receives the largest value of map t.
int run(const float* input, int batch, int sy, int sx, void* ws, size_t ws_bytes,
        const void* conv_data, float* output, int oy, int ox, int H, int W, bool conj,
        int device, void* stream, int* arg = nullptr, int tindex_base = 0, int reset = 0,
        float* sum = nullptr, float* sumsq = nullptr, float* peaks = nullptr) {
    g_last_error.clear();
    if (batch < 0) return fail(ZFFT_ERROR_INVALID_VALUE, "batch must be >= 0. Got %d.", batch);
    if (sy < 1 || sx < 1)
        return fail(ZFFT_ERROR_INVALID_VALUE, "signal lengths must be >= 1. Got (%d, %d).", sy, sx);
    if (!supported(H) || !supported(W))
        return fail(ZFFT_ERROR_UNSUPPORTED,
                    "Unsupported padded convolution configuration: signal_y=%d, signal_x=%d, "
                    "fft_y=%d, fft_x=%d, batch=%d, cross_correlate=%d (FFT sizes must be one of "
                    "64..4096 powers of two or 120, 240, 480, 960, 1920, 3840)",
                    sy, sx, H, W, batch, conj ? 1 : 0);
    if (sy > H || sx > W)
        return fail(ZFFT_ERROR_INVALID_VALUE,
                    "signal (%d, %d) larger than the FFT size (%d, %d)", sy, sx, H, W);
    const int vy = H - sy + 1, vx = W - sx + 1;
    const bool valid_out = (oy == vy && ox == vx);
    const bool full_out = (oy == H && ox == W);
    if (!valid_out && !full_out) {
        if (ox != vx && ox != W)
            return fail(ZFFT_ERROR_INVALID_VALUE,
                        "Output tensor last dimension must be fft_size_x - signal_length_x + 1 "
                        "(%d) or fft_size_x (%d). Got %d.",
                        vx, W, ox);
        return fail(ZFFT_ERROR_INVALID_VALUE,
                    "Output tensor second-to-last dimension must be fft_size_y - signal_length_y "
                    "+ 1 (%d) or fft_size_y (%d) matching the last dimension. Got %d.",
                    vy, H, oy);
    }
    const size_t need = zfft_workspace_bytes(H, W);
    if (ws_bytes < need)
        return fail(ZFFT_ERROR_INVALID_VALUE, "FFT workspace too small: %zu bytes, need %zu.",
                    ws_bytes, need);
    if (batch == 0) return ZFFT_SUCCESS;
    if (!input || !ws || !conv_data || !output)
        return fail(ZFFT_ERROR_INVALID_VALUE, "null data pointer");
    if (arg && !aligned(arg, 4)) return fail(ZFFT_ERROR_INVALID_VALUE, "misaligned argmax map");
    if ((sum && !aligned(sum, 4)) || (sumsq && !aligned(sumsq, 4)))
        return fail(ZFFT_ERROR_INVALID_VALUE, "misaligned sum map");
    if (peaks && !aligned(peaks, 4)) return fail(ZFFT_ERROR_INVALID_VALUE, "misaligned peaks");
    if (!aligned(input, 4) || !aligned(output, 4) || !aligned(ws, 16) || !aligned(conv_data, 16))
        return fail(ZFFT_ERROR_INVALID_VALUE,
                    "misaligned pointer: input/output need 4-byte alignment, fft_workspace and "
                    "conv_data 16-byte alignment (TMA copies)");
    int ndev = 0;
    cudaError_t e = device_count(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= ndev || device >= kMaxDevices)
        return fail(ZFFT_ERROR_INVALID_VALUE, "invalid device index %d (%d devices)", device, ndev);

    trace("call: batch %d signal (%d, %d) fft (%d, %d) out (%d, %d) conj %d device %d", batch,
          sy, sx, H, W, oy, ox, conj ? 1 : 0, device);
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return cuda_fail(guard.err, "cudaSetDevice");
    int rc = ensure_device(device);
    if (rc != ZFFT_SUCCESS) return rc;
    trace("device %d ready", device);

    const float2* pool = g_dev_pool[device];
    int* status = g_dev_status[device];
    const float2* twH = pool + tw_offset(H);
    const float2* twW = pool + tw_offset(W);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float2* Q = static_cast<float2*>(ws);
    const float2* spec = static_cast<const float2*>(conv_data);
    const int W2 = W / 2;
    const int nz_col = stage0_nz(H, sy);
    const int nz_row = stage0_nz(W2, (sx + 1) / 2);
    const float scale = float(1.0 / (double(H) * double(W)));

    // Workspace layout: Q (H x W2) first.  If the workspace holds more, the
    // row transforms of up to kMaxChunk templates run in one launch into a
    // region after Q (pitch h_pad); otherwise each template's rows go into
    // rows [0, h) of Q itself (pitch H).
    const long long h_pad = (sy + 1) / 2 * 2;
    const long long q_elems = (long long)H * W2;
    const long long r_elems = (long long)W2 * h_pad;
    const long long avail = (long long)(ws_bytes / sizeof(float2)) - q_elems;
    int chunk = 0;
    if (batch > 1 && avail >= r_elems) {
        const long long c = avail / r_elems;
        chunk = int(c < batch ? c : batch);
        if (chunk > kMaxChunk) chunk = kMaxChunk;
    }
    float2* Rregion = Q + q_elems;

    // Batched groups: when at least two whole Q slices fit in the workspace
    // (the reference's own (B, H, W/2+1) workspace holds B), up to kMaxChunk
    // templates go through each kernel in one launch, each in its own slice
    // (its row spectra first in rows [0, h) of the slice).  One launch per
    // kernel per group instead of one per template: no per-launch prologue
    // and tail per template, and the column pass reads each spectrum column
    // from DRAM once per group (neighbouring blocks share it in L2).  Measured
    // at 4096^2 / 32 x 256^2: 1.87 ms per call against 2.16 ms.  For the
    // running maps the inverse row pass also folds a row group's templates
    // one after another into map rows that stay in L2, instead of streaming
    // the whole maps through DRAM for every template.
    long long group = 0;
    if (batch > 1) {
        const long long fit_ws = (long long)(ws_bytes / sizeof(float2)) / q_elems;
        group = batch < fit_ws ? batch : fit_ws;
        if (group > kMaxChunk) group = kMaxChunk;
    }

    CUtensorMap qmap;
    e = qmap_fn(W)(Q, H, group >= 2 ? (int)group : 1, &qmap);
    if (e != cudaSuccess) return cuda_fail(e, "encoding the intermediate's tensor map");
    trace("tensor map encoded; chunk %d group %lld", chunk, group);
    ColFn col = col_fn(H);
    R2cFn r2c = r2c_fn(W);
    C2rFn c2r = c2r_fn(W);

    if (g_timer.on) g_timer.device = device;
    unsigned* peak_keys = reinterpret_cast<unsigned*>(peaks);
    if (peaks) {  // key 0 is below every value's key
        e = cudaMemsetAsync(peaks, 0, sizeof(float) * (size_t)batch, s);
        if (e != cudaSuccess) return cuda_fail(e, "clearing the peaks");
    }
    if (group >= 2) {
        for (int t0 = 0; t0 < batch; t0 += (int)group) {
            const int n = batch - t0 < group ? batch - t0 : (int)group;
            int m = timer_mark(s);
            e = r2c(input + (size_t)t0 * sy * sx, Q, twW, sy, sx, H, q_elems, n, scale, nz_row,
                    device, s);
            if (e != cudaSuccess) return cuda_fail(e, "row r2c launch");
            timer_close(0, m, s);
            if ((e = trace_sync(s, "k_row_r2c group", t0)) != cudaSuccess) return cuda_fail(e, "k_row_r2c");
            m = timer_mark(s);
            e = col(Q, Q, H, spec, twH, sy, W2, oy, conj, nz_col, false, n, q_elems, q_elems, status,
                    device, s);
            if (e != cudaSuccess) return cuda_fail(e, "column launch");
            timer_close(1, m, s);
            if ((e = trace_sync(s, "k_col_fused group", t0)) != cudaSuccess) return cuda_fail(e, "k_col_fused");
            m = timer_mark(s);
            if (arg)
                e = c2r(&qmap, output, arg, sum, sumsq, nullptr, twW, oy, ox, ox, tindex_base + t0,
                        t0 == 0 ? reset : 0, n, 0, status, device, s);
            else
                e = c2r(&qmap, output + (size_t)t0 * oy * ox, nullptr, nullptr, nullptr,
                        peak_keys ? peak_keys + t0 : nullptr, twW, oy, ox, ox, 0, 0, n,
                        (long long)oy * ox, status, device, s);
            if (e != cudaSuccess) return cuda_fail(e, "row c2r launch");
            timer_close(2, m, s);
            if ((e = trace_sync(s, "k_row_c2r group", t0)) != cudaSuccess) return cuda_fail(e, "k_row_c2r");
        }
    }
    const int step = chunk > 0 ? chunk : 1;
    for (int t0 = 0; group < 2 && t0 < batch; t0 += step) {
        const int n = batch - t0 < step ? batch - t0 : step;
        int m = -1;
        if (chunk > 0) {
            m = timer_mark(s);
            e = r2c(input + (size_t)t0 * sy * sx, Rregion, twW, sy, sx, (int)h_pad, r_elems, n,
                    scale, nz_row, device, s);
            if (e != cudaSuccess) return cuda_fail(e, "row r2c launch");
            timer_close(0, m, s);
            if ((e = trace_sync(s, "k_row_r2c chunk", t0)) != cudaSuccess) return cuda_fail(e, "k_row_r2c");
        }
        for (int j = 0; j < n; ++j) {
            const int t = t0 + j;
            const float2* Rt = Q;
            int r_pitch = H;
            if (chunk > 0) {
                Rt = Rregion + (size_t)j * r_elems;
                r_pitch = (int)h_pad;
            } else {
                m = timer_mark(s);
                e = r2c(input + (size_t)t * sy * sx, Q, twW, sy, sx, H, 0, 1, scale, nz_row, device, s);
                if (e != cudaSuccess) return cuda_fail(e, "row r2c launch");
                timer_close(0, m, s);
                if ((e = trace_sync(s, "k_row_r2c", t)) != cudaSuccess) return cuda_fail(e, "k_row_r2c");
            }
            m = timer_mark(s);
            e = col(Q, Rt, r_pitch, spec, twH, sy, W2, oy, conj, nz_col, chunk > 0, 1, 0, 0, status,
                    device, s);
            if (e != cudaSuccess) return cuda_fail(e, "column launch");
            timer_close(1, m, s);
            if ((e = trace_sync(s, "k_col_fused", t)) != cudaSuccess) return cuda_fail(e, "k_col_fused");
            m = timer_mark(s);
            if (arg)
                e = c2r(&qmap, output, arg, sum, sumsq, nullptr, twW, oy, ox, ox, tindex_base + t,
                        t == 0 ? reset : 0, 1, 0, status, device, s);
            else
                e = c2r(&qmap, output + (size_t)t * oy * ox, nullptr, nullptr, nullptr,
                        peak_keys ? peak_keys + t : nullptr, twW, oy, ox, ox, 0, 0, 1, 0, status,
                        device, s);
            if (e != cudaSuccess) return cuda_fail(e, "row c2r launch");
            timer_close(2, m, s);
            if ((e = trace_sync(s, "k_row_c2r", t)) != cudaSuccess) return cuda_fail(e, "k_row_c2r");
        }
    }
    if (peaks) {
        zf::k_peak_values<<<(batch + 255) / 256, 256, 0, s>>>(peak_keys, batch);
        if ((e = cudaGetLastError()) != cudaSuccess) return cuda_fail(e, "peak conversion launch");
    }
    return ZFFT_SUCCESS;
}

}  // namespace

namespace zf {

int plan_first_radix(int n) { return make_plan(n).R[0]; }

cudaError_t encode_tensor_map_2d(CUtensorMap* map, const void* base, unsigned long long dim0,
                                 unsigned long long dim1, unsigned long long stride1_bytes,
                                 unsigned box0, unsigned box1) {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static cudaError_t lookup_err = cudaSuccess;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        lookup_err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled",
                                             reinterpret_cast<void**>(&encode), cudaEnableDefault, &q);
        if (lookup_err == cudaSuccess && q != cudaDriverEntryPointSuccess)
            lookup_err = cudaErrorSymbolNotFound;
    });
    if (lookup_err != cudaSuccess) return lookup_err;
    cuuint64_t dims[2] = {dim0, dim1};
    cuuint64_t strides[1] = {stride1_bytes};
    cuuint32_t box[2] = {box0, box1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Bounded-wait self-test: the barrier expects 64 bytes but the single copy
// delivers 16, so the phase never completes; the wait must give up after
// `limit` cycles and report a timeout.  The copy itself has landed long
// before the limit, so nothing is in flight when the block exits.
__global__ void k_wait_selftest(int* status, long long limit) {
    __shared__ __align__(16) float4 dst[4];
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init_fence();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(&bar, 64);
        tma_load_1d(dst, &g_selftest_src, 16, &bar);
    }
    const bool ok = mbar_wait_bounded(&bar, 0, limit);
    if (__syncthreads_or(!ok) && threadIdx.x == 0) atomicExch(status, kStatusTimeout);
}

// Order-preserving 64-bit keys of (max, argmax) pairs for one integer MAX
// reduction across GPUs: high 32 bits = the float's bits mapped to unsigned
// order, low 32 bits = 0xFFFFFFFF - index (the lower index wins ties); the
// sign bit is flipped so that signed comparison (NCCL int64 MAX) orders keys
// like unsigned comparison.
__device__ __forceinline__ long long pack_key(float v, int idx) {
    uint32_t u = __float_as_uint(v);
    u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    const uint64_t k = (uint64_t(u) << 32) | uint64_t(0xFFFFFFFFu - uint32_t(idx));
    return (long long)(k ^ 0x8000000000000000ull);
}
__device__ __forceinline__ void unpack_key(long long key, float* v, int* idx) {
    const uint64_t k = uint64_t(key) ^ 0x8000000000000000ull;
    uint32_t u = uint32_t(k >> 32);
    u = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
    *v = __uint_as_float(u);
    *idx = int(0xFFFFFFFFu - uint32_t(k));
}
// Peaks: ordered keys (see ordered_key) -> float values, in place.
__global__ void k_peak_values(unsigned* keys, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) reinterpret_cast<float*>(keys)[i] = key_value(keys[i]);
}

__global__ void k_pack_keys(const float* __restrict__ v, const int* __restrict__ idx,
                            long long* __restrict__ keys, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        keys[i] = pack_key(v[i], idx[i]);
}
__global__ void k_unpack_keys(const long long* __restrict__ keys, float* __restrict__ v,
                              int* __restrict__ idx, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        unpack_key(keys[i], v + i, idx + i);
}

cudaError_t launch_wait_selftest(int* status, long long limit_cycles, cudaStream_t s) {
    k_wait_selftest<<<1, 32, 0, s>>>(status, limit_cycles);
    return cudaGetLastError();
}

}  // namespace zf

extern "C" {

int zfft_padded_real_corr_2d(const float* input, int batch, int signal_y, int signal_x,
                             void* fft_workspace, size_t fft_workspace_bytes,
                             const void* conv_data, float* output, int output_y, int output_x,
                             int fft_size_y, int fft_size_x, int device, void* stream) {
    return run(input, batch, signal_y, signal_x, fft_workspace, fft_workspace_bytes, conv_data,
               output, output_y, output_x, fft_size_y, fft_size_x, true, device, stream);
}

int zfft_padded_real_conv_2d(const float* input, int batch, int signal_y, int signal_x,
                             void* fft_workspace, size_t fft_workspace_bytes,
                             const void* conv_data, float* output, int output_y, int output_x,
                             int fft_size_y, int fft_size_x, int device, void* stream) {
    return run(input, batch, signal_y, signal_x, fft_workspace, fft_workspace_bytes, conv_data,
               output, output_y, output_x, fft_size_y, fft_size_x, false, device, stream);
}

size_t zfft_workspace_bytes(int fft_size_y, int fft_size_x) {
    if (!supported(fft_size_y) || !supported(fft_size_x)) return 0;
    return (size_t)fft_size_y * (size_t)(fft_size_x / 2) * sizeof(float2);
}

int zfft_is_fft_size_supported(int n) { return supported(n) ? 1 : 0; }

int zfft_get_supported_conv_configs(int* records, int capacity) {
    const int n = int(sizeof(kConfigs) / sizeof(kConfigs[0]));
    for (int i = 0; i < n && i < capacity && records; ++i)
        std::memcpy(records + 6 * i, kConfigs[i], sizeof(kConfigs[i]));
    return n;
}

const char* zfft_get_last_error(void) { return g_last_error.c_str(); }

int zfft_stage_timing_enable(int enable) {
    g_timer.on = enable != 0;
    return ZFFT_SUCCESS;
}

int zfft_stage_timing_read(double* ms, int* launches, int n) {
    if (n < kStages || !ms || !launches)
        return fail(ZFFT_ERROR_INVALID_VALUE, "stage timing needs arrays of %d entries", kStages);
    for (int st = 0; st < kStages; ++st) {
        ms[st] = 0.0;
        launches[st] = 0;
        for (auto& pr : g_timer.marks[st]) {
            cudaError_t e = cudaEventSynchronize(g_timer.pool[pr.second]);
            if (e != cudaSuccess) return cuda_fail(e, "stage timing event");
            float f = 0.f;
            e = cudaEventElapsedTime(&f, g_timer.pool[pr.first], g_timer.pool[pr.second]);
            if (e != cudaSuccess) return cuda_fail(e, "stage timing elapsed");
            ms[st] += f;
            launches[st] += 1;
        }
        g_timer.marks[st].clear();
    }
    g_timer.used = 0;
    return ZFFT_SUCCESS;
}

int zfft_get_version(void) { return kVersion; }

int zfft_image_spectrum(const float* image, int fft_size_y, int fft_size_x, void* conv_data,
                        size_t conv_data_bytes, int device, void* stream) {
    g_last_error.clear();
    const int H = fft_size_y, W = fft_size_x;
    if (!supported(H) || !supported(W))
        return fail(ZFFT_ERROR_UNSUPPORTED,
                    "Unsupported image size (%d, %d) (FFT sizes must be one of 64..4096 powers "
                    "of two or 120, 240, 480, 960, 1920, 3840)",
                    H, W);
    const size_t need = (size_t)(W / 2 + 1) * (size_t)H * sizeof(float2);
    if (conv_data_bytes < need)
        return fail(ZFFT_ERROR_INVALID_VALUE,
                    "conv_data too small: %zu bytes, need %zu ((W/2+1, H) complex64).",
                    conv_data_bytes, need);
    if (!image || !conv_data) return fail(ZFFT_ERROR_INVALID_VALUE, "null data pointer");
    if (!aligned(image, 4) || !aligned(conv_data, 16))
        return fail(ZFFT_ERROR_INVALID_VALUE,
                    "misaligned pointer: image needs 4-byte alignment, conv_data 16-byte "
                    "alignment (TMA copies)");
    int ndev = 0;
    cudaError_t e = device_count(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= ndev || device >= kMaxDevices)
        return fail(ZFFT_ERROR_INVALID_VALUE, "invalid device index %d (%d devices)", device, ndev);
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return cuda_fail(guard.err, "cudaSetDevice");
    int rc = ensure_device(device);
    if (rc != ZFFT_SUCCESS) return rc;
    const float2* pool = g_dev_pool[device];
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float2* spec = static_cast<float2*>(conv_data);
    // Row pass: every image row (full width, nothing pruned), unscaled,
    // column-major into the output itself (pitch H); then the column pass in
    // place.
    e = r2c_fn(W)(image, spec, pool + tw_offset(W), H, W, H, 0, 1, 1.0f, 0, device, s);
    if (e != cudaSuccess) return cuda_fail(e, "row r2c launch");
    if ((e = trace_sync(s, "k_row_r2c image", 0)) != cudaSuccess) return cuda_fail(e, "k_row_r2c");
    e = col_fwd_fn(H)(spec, pool + tw_offset(H), W / 2, g_dev_status[device], device, s);
    if (e != cudaSuccess) return cuda_fail(e, "column launch");
    if ((e = trace_sync(s, "k_col_fwd", 0)) != cudaSuccess) return cuda_fail(e, "k_col_fwd");
    return ZFFT_SUCCESS;
}

int zfft_padded_real_corr_2d_max(const float* input, int batch, int signal_y, int signal_x,
                                 void* fft_workspace, size_t fft_workspace_bytes,
                                 const void* conv_data, float* max_map, int32_t* arg_map,
                                 int output_y, int output_x, int fft_size_y, int fft_size_x,
                                 int template_index_base, int reset, int device, void* stream) {
    if (!arg_map && batch > 0) return fail(ZFFT_ERROR_INVALID_VALUE, "null argmax map");
    if (template_index_base < 0 || (long long)template_index_base + batch > 0x7FFFFFFFLL)
        return fail(ZFFT_ERROR_INVALID_VALUE, "template indices must lie in [0, 2^31 - 1)");
    return run(input, batch, signal_y, signal_x, fft_workspace, fft_workspace_bytes, conv_data,
               max_map, output_y, output_x, fft_size_y, fft_size_x, true, device, stream,
               reinterpret_cast<int*>(arg_map), template_index_base,
               reset != 0 ? zf::kResetMax : 0);
}

int zfft_padded_real_corr_2d_peaks(const float* input, int batch, int signal_y, int signal_x,
                                   void* fft_workspace, size_t fft_workspace_bytes,
                                   const void* conv_data, float* output, int output_y,
                                   int output_x, int fft_size_y, int fft_size_x, float* peaks,
                                   int device, void* stream) {
    if (!peaks && batch > 0) return fail(ZFFT_ERROR_INVALID_VALUE, "null peaks");
    return run(input, batch, signal_y, signal_x, fft_workspace, fft_workspace_bytes, conv_data,
               output, output_y, output_x, fft_size_y, fft_size_x, true, device, stream, nullptr, 0,
               false, nullptr, nullptr, peaks);
}

int zfft_padded_real_corr_2d_max_stats(const float* input, int batch, int signal_y,
                                       int signal_x, void* fft_workspace,
                                       size_t fft_workspace_bytes, const void* conv_data,
                                       float* max_map, int32_t* arg_map, float* sum_map,
                                       float* sumsq_map, int output_y, int output_x,
                                       int fft_size_y, int fft_size_x, int template_index_base,
                                       int reset, int device, void* stream) {
    if ((!arg_map || !sumsq_map) && batch > 0)
        return fail(ZFFT_ERROR_INVALID_VALUE, "null argmax or sum-of-squares map");
    if (template_index_base < 0 || (long long)template_index_base + batch > 0x7FFFFFFFLL)
        return fail(ZFFT_ERROR_INVALID_VALUE, "template indices must lie in [0, 2^31 - 1)");
    if (reset < 0 || reset > 2)
        return fail(ZFFT_ERROR_INVALID_VALUE,
                    "reset must be 0 (fold), 1 (overwrite every map) or 2 (overwrite the sum "
                    "maps only). Got %d.", reset);
    return run(input, batch, signal_y, signal_x, fft_workspace, fft_workspace_bytes, conv_data,
               max_map, output_y, output_x, fft_size_y, fft_size_x, true, device, stream,
               reinterpret_cast<int*>(arg_map), template_index_base,
               reset == 1 ? zf::kResetMax : (reset == 2 ? zf::kResetSums : 0), sum_map,
               sumsq_map);
}

namespace {
int launch_keys(bool pack, const float* v_in, float* v_out, const int32_t* i_in, int32_t* i_out,
                const int64_t* k_in, int64_t* k_out, size_t n, int device, void* stream) {
    g_last_error.clear();
    if (n == 0) return ZFFT_SUCCESS;
    int ndev = 0;
    cudaError_t e = device_count(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= ndev || device >= kMaxDevices)
        return fail(ZFFT_ERROR_INVALID_VALUE, "invalid device index %d (%d devices)", device, ndev);
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return cuda_fail(guard.err, "cudaSetDevice");
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    const long long blocks_needed = ((long long)n + 255) / 256;
    const int grid = (int)(blocks_needed < 8LL * sms ? blocks_needed : 8LL * sms);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (pack) {
        if (!v_in || !i_in || !k_out) return fail(ZFFT_ERROR_INVALID_VALUE, "null pointer");
        zf::k_pack_keys<<<grid, 256, 0, s>>>(v_in, reinterpret_cast<const int*>(i_in),
                                              reinterpret_cast<long long*>(k_out), (long long)n);
    } else {
        if (!k_in || !v_out || !i_out) return fail(ZFFT_ERROR_INVALID_VALUE, "null pointer");
        zf::k_unpack_keys<<<grid, 256, 0, s>>>(reinterpret_cast<const long long*>(k_in), v_out,
                                                reinterpret_cast<int*>(i_out), (long long)n);
    }
    e = cudaGetLastError();
    return e == cudaSuccess ? ZFFT_SUCCESS : cuda_fail(e, "key kernel launch");
}
}  // namespace

int zfft_pack_max_arg(const float* max_map, const int32_t* arg_map, int64_t* keys, size_t n,
                      int device, void* stream) {
    return launch_keys(true, max_map, nullptr, arg_map, nullptr, nullptr, keys, n, device, stream);
}

int zfft_unpack_max_arg(const int64_t* keys, float* max_map, int32_t* arg_map, size_t n, int device,
                        void* stream) {
    return launch_keys(false, nullptr, max_map, nullptr, arg_map, keys, nullptr, n, device, stream);
}

int zfft_padded_real_corr_2d_noalloc(const float* input, int batch, int signal_y, int signal_x,
                                     const void* conv_data, float* output, int output_y,
                                     int output_x, int fft_size_y, int fft_size_x, int device,
                                     void* stream) {
    g_last_error.clear();
    const size_t need = zfft_workspace_bytes(fft_size_y, fft_size_x);
    if (need == 0)
        return fail(ZFFT_ERROR_UNSUPPORTED,
                    "Unsupported padded convolution configuration: fft_y=%d, fft_x=%d",
                    fft_size_y, fft_size_x);
    if (need > kNoAllocBytes)
        return fail(ZFFT_ERROR_INVALID_VALUE,
                    "fft size (%d, %d) needs %zu bytes of scratch; the allocation-free entry "
                    "point has a fixed %zu-byte scratch array (fft_y * fft_x / 2 <= %zu); use "
                    "zfft_padded_real_corr_2d with a caller-provided workspace",
                    fft_size_y, fft_size_x, need, kNoAllocBytes, kNoAllocBytes / sizeof(float2));
    int ndev = 0;
    cudaError_t e = device_count(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= ndev || device >= kMaxDevices)
        return fail(ZFFT_ERROR_INVALID_VALUE, "invalid device index %d (%d devices)", device, ndev);
    // Set-up once per device, with that device current: the array's device
    // address (the symbol itself is only a host-side stand-in).
    static std::mutex mu;
    static float2* scratch[kMaxDevices];
    float2* ws = nullptr;
    {
        DeviceGuard guard(device);
        if (guard.err != cudaSuccess) return cuda_fail(guard.err, "cudaSetDevice");
        std::lock_guard<std::mutex> lock(mu);
        if (!scratch[device]) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_noalloc_ws);
            if (e != cudaSuccess) return cuda_fail(e, "resolving the fixed scratch array");
            scratch[device] = static_cast<float2*>(p);
        }
        ws = scratch[device];
    }
    return run(input, batch, signal_y, signal_x, ws, kNoAllocBytes, conv_data, output, output_y,
               output_x, fft_size_y, fft_size_x, true, device, stream);
}

int zfft_check_device_status(int device, void* stream, int* status) {
    g_last_error.clear();
    if (!status) return fail(ZFFT_ERROR_INVALID_VALUE, "status pointer is null");
    *status = ZFFT_SUCCESS;
    int ndev = 0;
    cudaError_t e = device_count(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= ndev || device >= kMaxDevices)
        return fail(ZFFT_ERROR_INVALID_VALUE, "invalid device index %d (%d devices)", device, ndev);
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return cuda_fail(guard.err, "cudaSetDevice");
    int rc = ensure_device(device);
    if (rc != ZFFT_SUCCESS) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
    int value = 0;
    e = cudaMemcpy(&value, g_dev_status[device], sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_fail(e, "reading the device status word");
    if (value != 0) {
        const int zero = 0;
        e = cudaMemcpy(g_dev_status[device], &zero, sizeof(int), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return cuda_fail(e, "clearing the device status word");
    }
    *status = value;
    return ZFFT_SUCCESS;
}

int zfft_selftest_wait_timeout(int device, void* stream) {
    g_last_error.clear();
    int ndev = 0;
    cudaError_t e = device_count(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= ndev || device >= kMaxDevices)
        return fail(ZFFT_ERROR_INVALID_VALUE, "invalid device index %d (%d devices)", device, ndev);
    DeviceGuard guard(device);
    if (guard.err != cudaSuccess) return cuda_fail(guard.err, "cudaSetDevice");
    int rc = ensure_device(device);
    if (rc != ZFFT_SUCCESS) return rc;
    // ~1 ms at 2 GHz
    trace("self-test launch");
    e = zf::launch_wait_selftest(g_dev_status[device], 2000000LL, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "self-test launch");
    if ((e = trace_sync(static_cast<cudaStream_t>(stream), "k_wait_selftest", 0)) != cudaSuccess)
        return cuda_fail(e, "k_wait_selftest");
    return ZFFT_SUCCESS;
}

}  // extern "C"
