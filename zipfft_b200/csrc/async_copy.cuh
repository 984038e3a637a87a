// Asynchronous global -> shared copies on sm_100a: TMA bulk (1D) and tensor
// (2D tile) loads completing on shared-memory mbarriers, and a bounded wait.
//
// No multicast form is used anywhere: every load fetches this GPU's own
// memory into the issuing block's shared memory.
//
// Every wait is bounded: after kWaitLimitCycles of polling the waiter gives
// up and the kernel reports ZFFT_ERROR_TIMEOUT through the device status word
// instead of hanging.
//
// Host compilation (the CPU test harness of the kernel logic) provides
// synchronous stand-ins with the same completion semantics.
#pragma once

#include <stdint.h>

#include "fft_core.cuh"

#if defined(__CUDACC__)
#include <cuda.h>  // CUtensorMap
#else
#include <chrono>
#include <cstring>
#include <vector>
#endif

namespace zf {

// Device status codes written by kernels (same values as the C ABI's).
constexpr int kStatusTimeout = 4;
// Bits of the running-map epilogues' `reset` argument (set by the C ABI).
constexpr int kResetMax = 1;   // overwrite every map (max, argmax, sums)
constexpr int kResetSums = 2;  // overwrite the sum maps only
// ~1 s at 2 GHz: far beyond any legitimate copy latency.
constexpr long long kWaitLimitCycles = 2000000000LL;

#if defined(__CUDACC__)

ZF_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

ZF_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Make barrier initialisation visible to the async (TMA) proxy.
ZF_DEV void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

ZF_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

ZF_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// L2 eviction-priority policies for cache-hinted accesses.
ZF_DEV uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
ZF_DEV uint64_t l2_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}
ZF_DEV uint64_t l2_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 1D bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned).
ZF_DEV void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
ZF_DEV void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2D tile load of the tensor map's box at (x, y); x * element size must be a
// multiple of 16 bytes.
ZF_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                        uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}

// 1D bulk store shared -> global (both addresses 16-byte aligned, bytes a
// multiple of 16), tracked as a bulk async-group of the issuing thread.
ZF_DEV void tma_store_1d(void* dst, const void* src, uint32_t bytes, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;" ::"l"(dst),
        "r"(smem_u32(src)), "r"(bytes), "l"(pol)
        : "memory");
}
ZF_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the issuing thread's bulk stores have finished reading shared
// memory (the source may then be overwritten).
ZF_DEV void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until the issuing thread's bulk stores have completed.
ZF_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Order this thread's generic shared-memory writes before later async-proxy
// reads of them (a bulk store issued after a barrier).
ZF_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Programmatic dependent launch: let the next kernel of the stream start its
// prologue while this one runs, and wait for the previous kernel's completion
// (and the visibility of its memory) before touching data it produced or
// still reads.  Both are no-ops for kernels launched without the attribute.
ZF_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
ZF_DEV void pdl_wait_prerequisites() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// 8-byte store with an L2 eviction policy.
ZF_DEV void st_hint(float2* p, float2 v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;" ::"l"(p), "f"(v.x),
                 "f"(v.y), "l"(pol)
                 : "memory");
}
ZF_DEV void st_hint(float* p, float v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(p), "f"(v), "l"(pol) : "memory");
}

// Drop a 128-byte L2 line without writing it back (its data becomes
// undefined).  `p` must be 128-byte aligned and no one may read the line again.
// Prefetch `bytes` (a multiple of 16) at the 16-byte aligned global address
// p into L2, asynchronously; nothing waits for it.
ZF_DEV void l2_prefetch_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

ZF_DEV void l2_discard_line(const void* p) {
    asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}

ZF_DEV long long cycle_clock() { return clock64(); }

#else  // host stand-ins for the CPU test harness -------------------------------

struct CUtensorMap {  // what the harness needs of a 2D tiled tensor map
    const unsigned char* base;
    long long dim0, dim1;  // elements
    long long stride1;     // bytes between dim-1 rows
    int box0, box1;
    int elem;  // bytes per element
};

// Barrier word: low 32 bits phase, high 32 bits outstanding bytes + arrivals.
void emu_mbar_init(uint64_t* bar, uint32_t count);
void emu_mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes);
void emu_mbar_complete_tx(uint64_t* bar, uint32_t bytes);
bool emu_mbar_try_wait(uint64_t* bar, uint32_t parity);

inline void mbar_init(uint64_t* bar, uint32_t count) { emu_mbar_init(bar, count); }
inline void mbar_init_fence() {}
inline void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    emu_mbar_arrive_expect_tx(bar, bytes);
}
inline bool mbar_try_wait(uint64_t* bar, uint32_t parity) { return emu_mbar_try_wait(bar, parity); }
void emu_check_copy(const void* dst, const void* src, uint32_t bytes);
// Delivers a TMA load's bytes (read from global memory at issue) into shared
// memory and completes them on the barrier: at once, or, in the harness's
// deferred mode, only when a thread next polls that barrier.
void emu_tma_arrive(void* dst, const void* data, uint32_t bytes, uint64_t* bar);
inline uint64_t l2_evict_first() { return 1; }
inline uint64_t l2_evict_last() { return 2; }
inline uint64_t l2_evict_normal() { return 3; }
inline void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t = 0) {
    emu_check_copy(dst, src, bytes);
    emu_tma_arrive(dst, src, bytes, bar);
}
void emu_check_store(const void* dst, const void* src, uint32_t bytes);
// A bulk store may read its shared-memory source at any time up to the
// issuing thread's wait: the harness records the source at issue and checks
// at the wait that nothing has written it since.
void emu_store_issued(const void* src, uint32_t bytes);
void emu_store_wait_read();
inline void tma_store_1d(void* dst, const void* src, uint32_t bytes, uint64_t) {
    emu_check_store(dst, src, bytes);
    std::memcpy(dst, src, bytes);
    emu_store_issued(src, bytes);
}
inline void pdl_launch_dependents() {}
inline void pdl_wait_prerequisites() {}
inline void bulk_commit() {}
inline void bulk_wait_read() { emu_store_wait_read(); }
inline void bulk_wait_all() { emu_store_wait_read(); }
inline void fence_proxy_async() {}
inline void st_hint(float2* p, float2 v, uint64_t) { *p = v; }
inline void st_hint(float* p, float v, uint64_t) { *p = v; }
void emu_check_prefetch(const void* p, uint32_t bytes);
inline void l2_prefetch_bulk(const void* p, uint32_t bytes) { emu_check_prefetch(p, bytes); }
void emu_discard_line(const void* p);
inline void l2_discard_line(const void* p) { emu_discard_line(p); }
inline void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                        uint64_t = 0) {
    const int row = map->box0 * map->elem;
    std::vector<unsigned char> tile((size_t)row * map->box1);
    unsigned char* d = tile.data();
    for (int j = 0; j < map->box1; ++j) {
        const long long yy = (long long)y + j;
        for (int i = 0; i < map->box0; ++i) {
            const long long xx = (long long)x + i;
            unsigned char* out = d + (size_t)j * row + (size_t)i * map->elem;
            if (xx < 0 || yy < 0 || xx >= map->dim0 || yy >= map->dim1) {
                std::memset(out, 0, map->elem);  // out-of-bounds fill
            } else {
                std::memcpy(out, map->base + yy * map->stride1 + xx * map->elem, map->elem);
            }
        }
    }
    emu_tma_arrive(dst, tile.data(), (uint32_t)tile.size(), bar);
}
inline long long cycle_clock() {  // nanoseconds stand in for cycles
    return (long long)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

#endif

// Bounded wait for the barrier phase with the given parity.
ZF_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                              long long limit = kWaitLimitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = cycle_clock();
    while (!mbar_try_wait(bar, parity)) {
        if (cycle_clock() - t0 > limit) return false;
    }
    return true;
}

}  // namespace zf
