// common.cuh -- shared helpers of the laprune_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "laprune_b200.h"

namespace lp {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_launch(const char* what);

#define LP_CHECK(cond, msg)                                  \
    do {                                                     \
        if (!(cond)) return ::lp::fail(LP_ERR_INVALID, msg); \
    } while (0)

#define LP_CUDA(call)                                                              \
    do {                                                                           \
        cudaError_t e_ = (call);                                                   \
        if (e_ != cudaSuccess)                                                     \
            return ::lp::fail(LP_ERR_CUDA, std::string(#call) + ": " +            \
                                               cudaGetErrorString(e_));            \
    } while (0)

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Carves consecutive 256-byte-aligned regions out of a workspace.
struct Carver {
    char* base;
    size_t off = 0;
    explicit Carver(void* b) : base(static_cast<char*>(b)) {}
    template <typename T>
    T* take(size_t count) {
        off = align_up(off, 256);
        T* p = reinterpret_cast<T*>(base ? base + off : nullptr);
        off += count * sizeof(T);
        return p;
    }
    size_t used() const { return align_up(off, 256); }
};

int sm_count(int device);

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
// Upper bound of any spin-wait, in SM clock cycles (about one second at the
// B200 boost clock); a wait that exceeds it records LP_DEVERR_WAIT_TIMEOUT
// and returns instead of hanging the GPU.
constexpr long long kWaitCycles = 2000000000LL;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

// Makes barrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false (and sets the error bit)
// if the phase did not complete within kWaitCycles.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > kWaitCycles) {
            if (err) atomicOr(err, LP_DEVERR_WAIT_TIMEOUT);
            return false;
        }
    }
    return true;
}

// 1-D bulk copy global -> shared (TMA engine), completion counted on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Same, with an L2 evict-first policy for data that is read exactly once.
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes,
                                                uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// Normal L2 priority, for streams that other CTAs read again soon after.
__device__ __forceinline__ uint64_t policy_evict_normal() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 16-byte asynchronous copy global -> shared (L2 only, bypassing L1).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// 4 consecutive codebook elements (fp32, or fp16 / bf16 widened exactly to
// fp32) at element index idx of a codebook of dtype dt (LP_F32 | LP_F16 |
// LP_BF16); idx a multiple of 4
__device__ __forceinline__ float4 cb_load4(const void* base, int64_t idx, int dt) {
    if (dt == LP_F32) return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(base) + idx));
    const uint2 raw = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(base) + idx));
    if (dt == LP_F16) {
        const __half2 a = *reinterpret_cast<const __half2*>(&raw.x), b = *reinterpret_cast<const __half2*>(&raw.y);
        return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
    }
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}
// the same from shared memory (a row staged by a bulk copy)
__device__ __forceinline__ float4 cb_lds4(const unsigned char* row, int i4, int dt) {
    if (dt == LP_F32) return reinterpret_cast<const float4*>(row)[i4];
    const uint2 raw = reinterpret_cast<const uint2*>(row)[i4];
    if (dt == LP_F16) {
        const __half2 a = *reinterpret_cast<const __half2*>(&raw.x), b = *reinterpret_cast<const __half2*>(&raw.y);
        return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
    }
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}
__host__ __device__ __forceinline__ int cb_elem_bytes(int dt) { return dt == LP_F32 ? 4 : 2; }

// Order-preserving map of an fp32 score into a histogram bin in [0, nb):
// bin = clamp(floor((s - lo) * inv_w)).  Monotone non-decreasing in s, so a
// token in a higher bin never has a lower score.  Written with explicit
// round-to-nearest intrinsics so every kernel computes the identical bin.
__device__ __forceinline__ int score_bin(float s, float lo, float inv_w, int nb) {
    float x = __fmul_rn(__fsub_rn(s, lo), inv_w);
    int b = __float2int_rd(x);  // NaN -> 0
    b = b < 0 ? 0 : b;
    return b >= nb ? nb - 1 : b;
}

}  // namespace lp
