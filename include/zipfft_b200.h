/* C ABI of libzipfft_b200.so: implicitly zero-padded real 2D FFT
 * convolution / cross-correlation on NVIDIA B200 (sm_100a).
 *
 * Every entry point takes plain pointers and sizes, launches asynchronously on
 * the given CUDA stream (a cudaStream_t passed as void*; NULL is the legacy
 * default stream) of the given device, and returns a status code.  On a
 * non-zero status zfft_get_last_error() describes the failure (per calling
 * thread).  Nothing here allocates device memory: all buffers are the
 * caller's.  The first call on a device uploads the twiddle tables (a
 * synchronous copy); make that first call outside CUDA graph capture.
 *
 * Reference interface replaced (mgiammar/zipFFT):
 *   src/cuda/real_conv_2d_binding.cu:288-299  conv / corr   (pybind11, torch::Tensor)
 *   src/cuda/real_conv_2d_binding.cu:189-285  padded_real_conv_2d_impl (validation + dispatch)
 *   src/cuda/real_conv_2d_binding.cu:160-170  get_supported_conv_configs
 *   src/cuda/real_conv_2d.cuh:296-335         padded_block_real_conv_2d (launcher)
 */
#ifndef ZIPFFT_B200_H_
#define ZIPFFT_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ZFFT_API __attribute__((visibility("default")))
#else
#define ZFFT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define ZFFT_SUCCESS 0
#define ZFFT_ERROR_INVALID_VALUE 1 /* bad shape, pointer, size or alignment */
#define ZFFT_ERROR_UNSUPPORTED 2   /* FFT size not built into the library */
#define ZFFT_ERROR_CUDA 3          /* CUDA runtime error (launch, device) */
#define ZFFT_ERROR_TIMEOUT 4       /* a bounded device-side wait gave up */

/* Padded real 2D convolution (conv) and cross-correlation (corr) of a batch of
 * small real templates with one large real image given by its spectrum.
 * Replaces zipfft.padded_rconv2d.conv / .corr (real_conv_2d_binding.cu:288-299).
 *
 *   input         float32 [batch][signal_y][signal_x], contiguous
 *   fft_workspace complex64 scratch, 16-byte aligned; at least
 *                 zfft_workspace_bytes(fft_y, fft_x) bytes (one
 *                 (fft_y, fft_x/2 + 1) slice, as in the reference, is always
 *                 enough; the reference's (batch, fft_y, fft_x/2 + 1) holds
 *                 one slice per template, and up to 32 templates then go
 *                 through each kernel per launch -- the fast choice).
 *                 Clobbered.
 *   conv_data     complex64 [fft_x/2 + 1][fft_y], 16-byte aligned: rfft2 of the
 *                 image, transposed (the reference's pre-transposed layout,
 *                 binding.cu:248-255)
 *   output        float32 [batch][output_y][output_x] where (output_y, output_x)
 *                 is either the valid crop (fft_y - signal_y + 1,
 *                 fft_x - signal_x + 1) as in the reference, or the full
 *                 circular map (fft_y, fft_x)
 *   fft_size_y/x  image size H, W (zfft_is_fft_size_supported)
 *
 * corr computes out[u][v] = sum_{y,x} T[y][x] I[(y+u) mod H][(x+v) mod W],
 * conv computes out[u][v] = sum_{y,x} T[y][x] I[(u-y) mod H][(v-x) mod W]
 * (torch.fft.irfftn(rfftn(I) * conj(rfftn(T, s=(H, W)))) and its unconjugated
 * form, norm="backward").  batch == 0 is a no-op. */
ZFFT_API int zfft_padded_real_corr_2d(const float* input, int batch, int signal_y, int signal_x,
                             void* fft_workspace, size_t fft_workspace_bytes,
                             const void* conv_data, float* output, int output_y, int output_x,
                             int fft_size_y, int fft_size_x, int device, void* stream);

ZFFT_API int zfft_padded_real_conv_2d(const float* input, int batch, int signal_y, int signal_x,
                             void* fft_workspace, size_t fft_workspace_bytes,
                             const void* conv_data, float* output, int output_y, int output_x,
                             int fft_size_y, int fft_size_x, int device, void* stream);

/* zfft_padded_real_corr_2d that also writes peaks[t] = the largest value of
 * output map t (batch float32 values, computed by the kernel that writes the
 * map, so no second pass over the output).  No counterpart in the reference;
 * the per-template best score of 2D template matching. */
ZFFT_API int zfft_padded_real_corr_2d_peaks(const float* input, int batch, int signal_y,
                                            int signal_x, void* fft_workspace,
                                            size_t fft_workspace_bytes, const void* conv_data,
                                            float* output, int output_y, int output_x,
                                            int fft_size_y, int fft_size_x, float* peaks,
                                            int device, void* stream);

/* 2D template matching's per-pixel search: cross-correlate every template
 * as zfft_padded_real_corr_2d does, but instead of writing one map per
 * template fold each correlation into running maps: max_map[y][x] keeps the
 * largest correlation seen and arg_map[y][x] the index of the template that
 * produced it (template t of this call has index template_index_base + t;
 * on ties the lower index is kept, since templates are folded in increasing
 * index order and only strictly larger values replace the maximum).  Both
 * maps are output_y x output_x (valid crop or full, as for corr).  reset != 0:
 * the call's first template overwrites the maps instead of comparing, so
 * they need no initialisation.  No counterpart in the reference (the fused
 * max / argmax of 2D template matching that its README motivates). */
ZFFT_API int zfft_padded_real_corr_2d_max(const float* input, int batch, int signal_y,
                                          int signal_x, void* fft_workspace,
                                          size_t fft_workspace_bytes, const void* conv_data,
                                          float* max_map, int32_t* arg_map, int output_y,
                                          int output_x, int fft_size_y, int fft_size_x,
                                          int template_index_base, int reset, int device,
                                          void* stream);

/* zfft_padded_real_corr_2d_max that also accumulates, per pixel, the sum and
 * the sum of squares of the correlations over the templates (float32 maps of
 * the same shape): the statistics 2D template matching normalises its scores
 * with.  reset: 0 folds every template into all four maps; 1 lets the first
 * template overwrite all four; 2 lets it overwrite the two sum maps only (the
 * maximum and argmax keep folding), so that a long search can sum each batch
 * in float32 and add the batches up at higher precision.  sum_map may be
 * NULL: the sum of squares alone is accumulated (the sum of a batch's maps is
 * also the map of the batch's summed template, correlation being linear, one
 * zfft_padded_real_corr_2d call).  No counterpart in the reference
 * (README.md:24 motivates the use). */
ZFFT_API int zfft_padded_real_corr_2d_max_stats(const float* input, int batch, int signal_y,
                                                int signal_x, void* fft_workspace,
                                                size_t fft_workspace_bytes, const void* conv_data,
                                                float* max_map, int32_t* arg_map, float* sum_map,
                                                float* sumsq_map, int output_y, int output_x,
                                                int fft_size_y, int fft_size_x,
                                                int template_index_base, int reset, int device,
                                                void* stream);

/* (max, argmax) pairs <-> one int64 key each, ordered so that a single
 * integer MAX reduction across GPUs (e.g. ncclAllReduce with ncclInt64 /
 * ncclMax) yields the global maximum and, on ties, the lowest index.  n
 * elements; asynchronous on `stream`.  No counterpart in the reference. */
ZFFT_API int zfft_pack_max_arg(const float* max_map, const int32_t* arg_map, int64_t* keys,
                               size_t n, int device, void* stream);
ZFFT_API int zfft_unpack_max_arg(const int64_t* keys, float* max_map, int32_t* arg_map, size_t n,
                                 int device, void* stream);

/* Cross-correlation exactly as zfft_padded_real_corr_2d, for callers that
 * cannot allocate device memory.  No counterpart in the reference (whose
 * binding takes a caller-allocated workspace tensor).  Instead of a workspace
 * argument it uses a fixed 16 MiB scratch array that lives in the library's
 * own device memory: every GPU that loads the library holds it until the
 * process exits.  Limit: fft_y * (fft_x / 2) complex values must fit, i.e.
 * fft_y * fft_x <= 4,194,304 (e.g. 2048 x 2048, 4096 x 1024); larger sizes
 * return ZFFT_ERROR_INVALID_VALUE with an explanation.  The call itself makes
 * no cudaMalloc / cudaFree or other allocating call.  The first call on a
 * device looks the array's device address up (and uploads the twiddle tables,
 * as every first call does); make that first call before any stream capture.
 * All calls share the one array and it keeps the previous call's contents
 * (nothing in it needs to start at zero): calls that can overlap on the GPU
 * (different streams, or different host threads without ordering) race on it
 * and give wrong results; serialize them. */
ZFFT_API int zfft_padded_real_corr_2d_noalloc(const float* input, int batch, int signal_y,
                                              int signal_x, const void* conv_data, float* output,
                                              int output_y, int output_x, int fft_size_y,
                                              int fft_size_x, int device, void* stream);

/* Bytes of fft_workspace that zfft_padded_real_corr_2d, _conv_2d, _corr_2d_max,
 * _corr_2d_peaks and _corr_2d_max_stats need for an (fft_y, fft_x) image:
 * fft_y * (fft_x / 2) complex64 values, independent of the batch (templates
 * then go one after another through the same slice; each further whole slice
 * lets one more template share the launches, up to 32).
 * Returns 0 for unsupported sizes.  No counterpart in the reference, which
 * sizes the workspace (batch, fft_y, fft_x/2 + 1) (binding.cu:235-245). */
ZFFT_API size_t zfft_workspace_bytes(int fft_size_y, int fft_size_x);

/* 1 if n is a supported FFT size (for H and W), else 0.  Replaces the
 * compile-time shape table's size check (binding.cu:51-106). */
ZFFT_API int zfft_is_fft_size_supported(int n);

/* Validated configurations as 6-int records (signal_y, signal_x, fft_y, fft_x,
 * batch, cross_correlate); writes at most `capacity` records and returns the
 * total count.  Replaces get_supported_conv_configs (binding.cu:160-170). */
ZFFT_API int zfft_get_supported_conv_configs(int* records, int capacity);

/* Description of the last failure on the calling thread ("" if none). */
ZFFT_API const char* zfft_get_last_error(void);

/* Per-stage device timing for benchmarks (no counterpart in the reference,
 * whose benchmark times whole calls: benchmark/run_benchmark.cu:364-379).
 * While enabled on the calling thread, every kernel launch of the calls above
 * is bracketed by CUDA events on the call's stream.  zfft_stage_timing_read
 * waits for those events and writes, for stage 0 (row r2c), 1 (fused column)
 * and 2 (row c2r), the summed milliseconds and launch counts (arrays of n >= 3
 * entries), then clears the record. */
ZFFT_API int zfft_stage_timing_enable(int enable);
ZFFT_API int zfft_stage_timing_read(double* ms, int* launches, int n);

/* Device status: kernels never spin without bound.  Every wait on an
 * asynchronous copy gives up after about a second; the kernel then records
 * ZFFT_ERROR_TIMEOUT in a per-device status word and exits instead of hanging
 * the GPU.  zfft_check_device_status synchronizes `stream`, stores the word
 * (0 = no failure since the last check) in *status and clears it.  No
 * counterpart in the reference, whose launcher only checks launch errors
 * (real_conv_2d.cuh:279-289). */
ZFFT_API int zfft_check_device_status(int device, void* stream, int* status);

/* Runs a one-block kernel whose wait can never complete (its barrier expects
 * more bytes than its copy delivers) with a ~1 ms limit, so that the timeout
 * path can be exercised: afterwards zfft_check_device_status reports
 * ZFFT_ERROR_TIMEOUT.  For tests. */
ZFFT_API int zfft_selftest_wait_timeout(int device, void* stream);

/* Image spectrum in the layout conv_data takes: the 2D real FFT of the
 * (fft_y, fft_x) float32 image (row-major, contiguous), unnormalised,
 * transposed to (fft_x/2 + 1, fft_y) complex64, i.e. element (kx, ky) at
 * kx * fft_y + ky.  Replaces the caller-side torch.fft.rfftn(image)
 * .transpose(-2, -1) that the reference's users run before calling the
 * operator (README.md:224-228; tests/test_real_conv_2d.py:89-90, :125-127);
 * the reference has no entry point for it.  conv_data_bytes must be at least
 * (fft_x/2 + 1) * fft_y * 8; conv_data needs 16-byte alignment.  Uses no
 * other memory (the row transforms are staged in conv_data itself) and, like
 * the calls above, runs asynchronously on `stream`. */
ZFFT_API int zfft_image_spectrum(const float* image, int fft_size_y, int fft_size_x,
                                 void* conv_data, size_t conv_data_bytes, int device,
                                 void* stream);

/* Library version as major * 10000 + minor * 100 + patch. */
ZFFT_API int zfft_get_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ZIPFFT_B200_H_ */
