// icm.cuh -- ICM refinement of greedy additive-quantization codes.
//
// Reference: laprune/quantizer.py:356-370 (the loop of _batch_icm_lut after
// its greedy pass), reached from AQLayerCodebookManager.encode_keys(_batch)
// (laprune/llm/aq_kv.py:348-429, default icm_iters=2) and from
// AdditiveQuantizer.encode (quantizer.py:319-344).  After the greedy pass,
// full_recon = x - r; each sweep re-chooses code m = 0..31 of every vector:
//     recon_wo = full_recon - C_m[prev];  r = x - recon_wo;
//     new = first argmin_k ||r||^2 + ||C_m[k]||^2 - 2 r.C_m[k];
//     full_recon = recon_wo + C_m[new]
// and a sweep that changes no code of the batch (the vectors that share a
// codebook set: the reference runs one quantizer per codebook group) ends the
// refinement.  One launch per sweep: a launch reads the previous sweep's
// count of changed codes of its set and returns at once when it is zero.
//
// Arithmetic (the same as the greedy encoder's and the oracle's): elementwise
// fp32 subtractions and additions as written above; ||r||^2 a sequential fma
// chain in index order; r.c as 32 four-term fma chains over dims 4l..4l+3
// folded by a butterfly at strides 16, 8, 4, 2, 1; dist = fma(-2, r.c,
// ||r||^2 + ||c||^2); the smallest (distance, codeword) wins.  All on CUDA
// cores: this refinement is off the decode path (the decode configurations
// encode greedily), so it is written for exactness first.
//
// Work split: a CTA holds 4 vectors; warp w serves vector w / 4 and the 64
// codewords 64 (w % 4) .. +63 of every stage; lane l holds dims 4l..4l+3 of
// its vector's x, reconstruction and residual in registers.  The 4 warps of
// a vector combine their smallest keys through shared memory once per stage.
#pragma once
#include "common.cuh"
#include "encode.cuh"

namespace lp {

constexpr int kIcmThreads = 512;
constexpr int kIcmVec = 4;  // vectors per CTA (4 warps each)

struct IcmParams {
    const void* x;
    int64_t xs_b, xs_h, xs_t;  // elements
    int B, H, T;               // vectors x[b][h][t][0..128)
    int per_head;              // codebook set of vector (b, h, t) is h (else 0)
    const float* cb;           // [S][32][256][128] fp32
    const float* nrm;          // [S][32][256] ||C||^2 (sequential fma)
    uint8_t* codes;            // greedy codes on entry of sweep 0, refined in place
    int64_t cs_b, cs_h, cs_t;  // bytes
    float* fr;                 // [S][vectors of a set][128] reconstruction between sweeps
    uint32_t* changed;         // [sweeps][S] codes changed by each sweep (zeroed before sweep 0)
    int sweep;                 // this launch's sweep, 0-based
    int last;                  // the last sweep: the reconstruction is not stored
    int ctas_per_set;
    uint32_t* err;
};

template <typename XT>
__global__ void __launch_bounds__(kIcmThreads) icm_sweep_kernel(IcmParams p) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int set = blockIdx.x / p.ctas_per_set;
    const int tile = blockIdx.x - set * p.ctas_per_set;
    const int nsets = gridDim.x / p.ctas_per_set;
    // the set's refinement ended when the previous sweep changed nothing
    // (quantizer.py:368-369); uniform over the CTA
    if (p.sweep > 0 && __ldcg(p.changed + (int64_t)(p.sweep - 1) * nsets + set) == 0u) return;

    const int vi = warp >> 2, qtr = warp & 3;
    const int nvec_set = p.per_head ? p.B * p.T : p.B * p.H * p.T;
    const int v = tile * kIcmVec + vi;
    const bool live = v < nvec_set;  // warp-uniform
    const float* cbs = p.cb + (int64_t)set * kEncM * kEncK * kEncD;
    const float* nrs = p.nrm + (int64_t)set * kEncM * kEncK;
    __shared__ unsigned long long s_key[2][kIcmVec][4];
    __shared__ uint8_t s_codes[kIcmVec][kEncM];
    __shared__ uint32_t s_changed;

    float4 xv = make_float4(0.f, 0.f, 0.f, 0.f), fr = xv;
    uint8_t* cod = nullptr;
    if (live) {
        int b, h, t;
        if (p.per_head) {
            h = set;
            b = v / p.T;
            t = v - b * p.T;
        } else {
            const int ht = p.H * p.T;
            b = v / ht;
            const int r = v - b * ht;
            h = r / p.T;
            t = r - h * p.T;
        }
        const XT* xr = reinterpret_cast<const XT*>(p.x) + (int64_t)b * p.xs_b + (int64_t)h * p.xs_h +
                       (int64_t)t * p.xs_t + 4 * lane;
        xv = make_float4(to_f32(xr[0]), to_f32(xr[1]), to_f32(xr[2]), to_f32(xr[3]));
        cod = p.codes + (int64_t)b * p.cs_b + (int64_t)h * p.cs_h + (int64_t)t * p.cs_t;
        if (qtr == 0) s_codes[vi][lane] = cod[lane];
    }
    if (tid == 0) s_changed = 0u;
    __syncthreads();
    auto cw4 = [&](int m, int k) -> float4 {  // dims 4 lane .. +3 of C_m[k]
        return __ldg(reinterpret_cast<const float4*>(cbs + ((int64_t)m * kEncK + k) * kEncD) + lane);
    };
    if (live) {
        if (p.sweep == 0) {
            // the greedy residual r = x - sum_m C_m[code_m] (in stage order),
            // then full_recon = x - r
            float4 r = xv;
#pragma unroll 8
            for (int m = 0; m < kEncM; ++m) {
                const float4 c = cw4(m, s_codes[vi][m]);
                r.x = __fsub_rn(r.x, c.x);
                r.y = __fsub_rn(r.y, c.y);
                r.z = __fsub_rn(r.z, c.z);
                r.w = __fsub_rn(r.w, c.w);
            }
            fr = make_float4(__fsub_rn(xv.x, r.x), __fsub_rn(xv.y, r.y), __fsub_rn(xv.z, r.z), __fsub_rn(xv.w, r.w));
        } else {
            fr = __ldcg(reinterpret_cast<const float4*>(p.fr + ((int64_t)set * nvec_set + v) * kEncD) + lane);
        }
    }
    uint32_t nch = 0u;
    for (int m = 0; m < kEncM; ++m) {
        unsigned long long best = ~0ull;
        float4 rw = fr;
        int prev = 0;
        if (live) {
            prev = s_codes[vi][m];
            const float4 cp = cw4(m, prev);
            rw = make_float4(__fsub_rn(fr.x, cp.x), __fsub_rn(fr.y, cp.y), __fsub_rn(fr.z, cp.z), __fsub_rn(fr.w, cp.w));
            const float4 r =
                make_float4(__fsub_rn(xv.x, rw.x), __fsub_rn(xv.y, rw.y), __fsub_rn(xv.z, rw.z), __fsub_rn(xv.w, rw.w));
            // ||r||^2: one chain over dims 0..127, lane by lane
            float rn = 0.f;
#pragma unroll 8
            for (int L = 0; L < 32; ++L) {
                const float a = __shfl_sync(0xffffffffu, r.x, L), b = __shfl_sync(0xffffffffu, r.y, L);
                const float c = __shfl_sync(0xffffffffu, r.z, L), d = __shfl_sync(0xffffffffu, r.w, L);
                rn = __fmaf_rn(a, a, rn);
                rn = __fmaf_rn(b, b, rn);
                rn = __fmaf_rn(c, c, rn);
                rn = __fmaf_rn(d, d, rn);
            }
            const float* nm = nrs + (int64_t)m * kEncK + qtr * 64;
#pragma unroll 4
            for (int kk = 0; kk < 64; ++kk) {
                const int k = qtr * 64 + kk;
                const float4 c = cw4(m, k);
                float dot = __fmaf_rn(r.x, c.x, 0.f);
                dot = __fmaf_rn(r.y, c.y, dot);
                dot = __fmaf_rn(r.z, c.z, dot);
                dot = __fmaf_rn(r.w, c.w, dot);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) dot = __fadd_rn(dot, __shfl_xor_sync(0xffffffffu, dot, o));
                // +0 folds a -0 into +0, so that equal distances have equal keys
                const float dist = __fadd_rn(__fmaf_rn(-2.f, dot, __fadd_rn(rn, __ldg(nm + kk))), 0.f);
                uint32_t key = __float_as_uint(dist);
                key = (key & 0x80000000u) ? ~key : (key | 0x80000000u);  // float order as unsigned order
                const unsigned long long kv = ((unsigned long long)key << 32) | (unsigned)k;
                best = kv < best ? kv : best;
            }
        }
        if (lane == 0) s_key[m & 1][vi][qtr] = best;
        __syncthreads();
        if (live) {
            unsigned long long b0 = s_key[m & 1][vi][0];
#pragma unroll
            for (int j = 1; j < 4; ++j) b0 = s_key[m & 1][vi][j] < b0 ? s_key[m & 1][vi][j] : b0;
            const int nw = (int)(b0 & 0xffu);
            if (qtr == 0 && lane == 0) {
                nch += nw != prev ? 1u : 0u;
                s_codes[vi][m] = (uint8_t)nw;  // read by the other warps only before this stage's barrier
            }
            const float4 cn = cw4(m, nw);
            fr = make_float4(__fadd_rn(rw.x, cn.x), __fadd_rn(rw.y, cn.y), __fadd_rn(rw.z, cn.z), __fadd_rn(rw.w, cn.w));
        }
    }
    if (live) {
        if (!p.last) reinterpret_cast<float4*>(p.fr + ((int64_t)set * nvec_set + v) * kEncD)[lane] = fr;
        if (qtr == 0) {
            __syncwarp();
            cod[lane] = s_codes[vi][lane];
            if (lane == 0 && nch) atomicAdd(&s_changed, nch);
        }
    }
    __syncthreads();
    if (tid == 0 && s_changed) atomicAdd(p.changed + (int64_t)p.sweep * nsets + set, s_changed);
}

}  // namespace lp
