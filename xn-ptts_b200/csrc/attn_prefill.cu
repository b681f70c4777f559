// Causal attention for rows that sit anywhere in their stream (a prompt, or several rows of a
// host-position step): row r of a stream at position p attends keys 0..=p of that stream.
//
// Reference: the t > 1 branch of StreamingMultiheadAttention::forward (transformer.rs:231-248),
// softmax(q k^T * 1/sqrt(d) + mask) v with the mask of materialize_causal_mask
// (transformer.rs:94-108): key k visible to query q iff k <= q + current_end.
//
// One warp per (row, head), CUDA cores: 8 lanes cover one 128-byte head row, 4 keys per warp
// instruction, keys read straight from the cache (coalesced 128-byte segments), online softmax
// in the exp2 domain as in the decode kernel.
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int kHeads = kRowWidth / kHeadDim;

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void load8g(const __nv_bfloat16* p, int j, float* o) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p) + j);
    o[0] = bf16lo(u.x); o[1] = bf16hi(u.x); o[2] = bf16lo(u.y); o[3] = bf16hi(u.y);
    o[4] = bf16lo(u.z); o[5] = bf16hi(u.z); o[6] = bf16lo(u.w); o[7] = bf16hi(u.w);
}
__device__ __forceinline__ void load8g(const float* p, int j, float* o) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p) + j);
    const float4 b = __ldg(reinterpret_cast<const float4*>(p + 32) + j);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
template <typename T>
__device__ __forceinline__ int dim_of(int j, int i) {
    if (sizeof(T) == 2) return 8 * j + i;
    return i < 4 ? 4 * j + i : 32 + 4 * j + (i - 4);
}

template <typename T>
__global__ void __launch_bounds__(256) prefill_attn_kernel(PrefillArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (w >= a.rows * kHeads) return;
    const int row = w / kHeads, h = w % kHeads;
    const int g = lane >> 3, j = lane & 7;
    const int sid = a.row_stream[row];
    const int pos = a.row_pos[row];
    const long long cap_rows = a.stream_elems / kRowWidth;
    // Keys: positions first..pos; a windowed stream keeps its last `context` (Mimi's mask,
    // transformer.rs:762-785: 0 <= pos - key < context) at slots modulo the capacity.
    const int ctx = a.window ? a.window[sid] : 0;
    const int first = ctx > 0 ? max(0, pos - ctx + 1) : 0;
    const int nk = pos - first + 1;
    if (sid < 0 || pos < 0 || nk > cap_rows || (ctx == 0 && pos + 1 > cap_rows)) {
        set_error(a.err, DEV_ERR_BOUNDS);
        return;
    }
    const T* kb = static_cast<const T*>(a.k_cache) + (long long)sid * a.stream_elems + h * kHeadDim;
    const T* vb = static_cast<const T*>(a.v_cache) + (long long)sid * a.stream_elems + h * kHeadDim;
    float q[8];
    {
        const float* qh = a.q + (long long)row * a.ld + h * kHeadDim;
        const float4 x = *reinterpret_cast<const float4*>(qh + (sizeof(T) == 2 ? 8 * j : 4 * j));
        const float4 y = *reinterpret_cast<const float4*>(qh + (sizeof(T) == 2 ? 8 * j + 4 : 32 + 4 * j));
        q[0] = x.x; q[1] = x.y; q[2] = x.z; q[3] = x.w;
        q[4] = y.x; q[5] = y.y; q[6] = y.z; q[7] = y.w;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] *= a.qscale;
    float m = -1e30f, l = 0.f, acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
    for (int r = 0; r < nk; r += 8) {
        const int r0 = r + g, r1 = r + 4 + g;
        const int rr0 = r0 < nk ? r0 : nk - 1, rr1 = r1 < nk ? r1 : nk - 1;
        float k0[8], k1[8], v0[8], v1[8];
        const long long sl0 = (first + rr0) % cap_rows, sl1 = (first + rr1) % cap_rows;
        load8g(kb + sl0 * kRowWidth, j, k0);
        load8g(kb + sl1 * kRowWidth, j, k1);
        load8g(vb + sl0 * kRowWidth, j, v0);
        load8g(vb + sl1 * kRowWidth, j, v1);
        float d0 = 0.f, d1 = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            d0 = fmaf(q[i], k0[i], d0);
            d1 = fmaf(q[i], k1[i], d1);
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            d0 += __shfl_xor_sync(0xffffffffu, d0, o);
            d1 += __shfl_xor_sync(0xffffffffu, d1, o);
        }
        if (r0 >= nk) d0 = -INFINITY;
        if (r1 >= nk) d1 = -INFINITY;
        const float mn = fmaxf(m, fmaxf(d0, d1));
        const float corr = fast_exp2(m - mn);
        const float e0 = fast_exp2(d0 - mn), e1 = fast_exp2(d1 - mn);
        l = fmaf(l, corr, e0 + e1);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = fmaf(e1, v1[i], fmaf(e0, v0[i], acc[i] * corr));
        m = mn;
    }
#pragma unroll
    for (int o = 8; o <= 16; o <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, o);
        const float lo = __shfl_xor_sync(0xffffffffu, l, o);
        const float mn = fmaxf(m, mo);
        const float fa = fast_exp2(m - mn), fb = fast_exp2(mo - mn);
        l = l * fa + lo * fb;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = acc[i] * fa + __shfl_xor_sync(0xffffffffu, acc[i], o) * fb;
        m = mn;
    }
    if (g != 0) return;
    const float inv = 1.f / l;
    const long long at = (long long)row * a.ld + h * kHeadDim;
    if (a.out_mode == kOutF32) {
        float* o = static_cast<float*>(a.out) + at;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[dim_of<T>(j, i)] = acc[i] * inv;
    } else if (a.out_mode == kOutBf16) {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + at;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[dim_of<T>(j, i)] = __float2bfloat16_rn(acc[i] * inv);
    } else {
        __half* o = static_cast<__half*>(a.out) + at;
        __half* ol = static_cast<__half*>(a.out_lo) + at;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float hf, lf;
            split_f16(acc[i] * inv, hf, lf);
            o[dim_of<T>(j, i)] = __float2half_rn(hf);
            ol[dim_of<T>(j, i)] = __float2half_rn(lf);
        }
    }
}

}  // namespace

void launch_prefill_attn(const PrefillArgs& a, bool cache_bf16, cudaStream_t s) {
    const int blocks = (a.rows * kHeads + 7) / 8;
    if (cache_bf16) launch_k(prefill_attn_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, a);
    else launch_k(prefill_attn_kernel<float>, dim3(blocks), dim3(256), 0, s, a);
}

}  // namespace ptts
