// rope_append.cuh -- one decode token: rotary position embedding of its query
// and key rows, fused with the append of the rotated key and the value to a
// preallocated (static) K/V cache.
//
// Reference: laprune/llm/modifiers/aq_evaluation.py:296-308 (self_attn_forward:
// HF apply_rotary_pos_emb on q and k, then _kv_cache_append's slice copies
// into the growable cache, :65-112).  The rotation is HF's
//     x_rot = x * cos + rotate_half(x) * sin,  rotate_half(x) = [-x2, x1]
// with each product and the sum rounded to the tensor dtype as PyTorch's
// elementwise ops on bf16/fp16 tensors do (fp32 arithmetic, one rounding per
// op), so the rows equal the reference's bit for bit.
#pragma once
#include "common.cuh"

namespace lp {

struct RopeAppendParams {
    const void* q;
    const void* k;
    const void* v;
    int64_t q_sb, q_sh, k_sb, k_sh, v_sb, v_sh;
    const void* cos;
    const void* sin;
    int64_t cos_sb, sin_sb;
    void* q_out;
    int64_t qo_sb, qo_sh;
    void* k_cache;
    void* v_cache;
    int64_t kc_sb, kc_sh, kc_st, vc_sb, vc_sh, vc_st;
    int Hq, Hkv, D, pos;
};

// round-to-dtype of an fp32 value, back in fp32
template <typename T>
__device__ __forceinline__ float round_to(float x) {
    return to_f32<T>(from_f32<T>(x));
}

// grid (rows = Hq + 2 Hkv, B), D/2 threads: thread i rotates the pair
// (i, i + D/2) of its row; value rows are copied
template <typename T>
__global__ void rope_append_kernel(RopeAppendParams p) {
    const int row = blockIdx.x, b = blockIdx.y, i = threadIdx.x;
    const int half = p.D / 2;
    if (i >= half) return;
    if (row >= p.Hq + p.Hkv) {  // value row: plain append
        const int h = row - p.Hq - p.Hkv;
        const T* src = reinterpret_cast<const T*>(p.v) + (int64_t)b * p.v_sb + (int64_t)h * p.v_sh;
        T* dst = reinterpret_cast<T*>(p.v_cache) + (int64_t)b * p.vc_sb + (int64_t)h * p.vc_sh + (int64_t)p.pos * p.vc_st;
        dst[i] = src[i];
        dst[i + half] = src[i + half];
        return;
    }
    const bool is_q = row < p.Hq;
    const int h = is_q ? row : row - p.Hq;
    const T* src = is_q ? reinterpret_cast<const T*>(p.q) + (int64_t)b * p.q_sb + (int64_t)h * p.q_sh
                        : reinterpret_cast<const T*>(p.k) + (int64_t)b * p.k_sb + (int64_t)h * p.k_sh;
    T* dst = is_q ? reinterpret_cast<T*>(p.q_out) + (int64_t)b * p.qo_sb + (int64_t)h * p.qo_sh
                  : reinterpret_cast<T*>(p.k_cache) + (int64_t)b * p.kc_sb + (int64_t)h * p.kc_sh +
                        (int64_t)p.pos * p.kc_st;
    const T* cs = reinterpret_cast<const T*>(p.cos) + (int64_t)b * p.cos_sb;
    const T* sn = reinterpret_cast<const T*>(p.sin) + (int64_t)b * p.sin_sb;
    const float x1 = to_f32(src[i]), x2 = to_f32(src[i + half]);
    // out[i] = x1 cos[i] + (-x2) sin[i];  out[i + half] = x2 cos[i + half] + x1 sin[i + half]
    const float a = round_to<T>(__fmul_rn(x1, to_f32(cs[i])));
    const float c = round_to<T>(__fmul_rn(-x2, to_f32(sn[i])));
    const float e = round_to<T>(__fmul_rn(x2, to_f32(cs[i + half])));
    const float f = round_to<T>(__fmul_rn(x1, to_f32(sn[i + half])));
    dst[i] = from_f32<T>(__fadd_rn(a, c));
    dst[i + half] = from_f32<T>(__fadd_rn(e, f));
}

}  // namespace lp
