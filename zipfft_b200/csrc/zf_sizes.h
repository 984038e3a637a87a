// FFT sizes (image height H and width W) the library is built for.  Any
// template size h <= H, w <= W and any batch works at run time; only the FFT
// sizes are compile-time, each one instantiating its own kernels.
//   powers of two 64 .. 4096, and 15 * 2^k sizes 120 .. 3840 (radix-3/5 path).
#pragma once

#define ZF_FOR_EACH_FFT_SIZE(X) \
    X(64)                       \
    X(128)                      \
    X(256)                      \
    X(512)                      \
    X(1024)                     \
    X(2048)                     \
    X(4096)                     \
    X(120)                      \
    X(240)                      \
    X(480)                      \
    X(960)                      \
    X(1920)                     \
    X(3840)

// Sum of all sizes: the twiddle pool holds one table of N roots per size.
#define ZF_TW_POOL_TOTAL (64 + 128 + 256 + 512 + 1024 + 2048 + 4096 + 120 + 240 + 480 + 960 + 1920 + 3840)
