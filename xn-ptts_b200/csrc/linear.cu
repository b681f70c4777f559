// int8-weight linears of the flow-LM layer with their neighbours fused in.
//
// Reference: Q::LinearQ::forward for in_proj, out_proj, linear1 and linear2
// (ptts/src/transformer.rs:195, :224, :627) around LayerNorm (:602, :618), GELU (:620-625) and
// the residual adds (:616, :634). Weights are int8 [out][in] with one f32 scale per output row,
// so y[m][n] = scale[n] * sum_k a[m][k] * q[n][k]; int8 values are exact in bf16, so the
// products run on the tensor cores with the scale applied once in the epilogue.
//
// Prologues:  plain   A = bf16 rows from global memory, streamed with B;
//             ln      A = LayerNorm(x) of f32 residual rows, computed once per CTA into a
//                     resident bf16 tile (transformer.rs:547-548, eps 1e-5).
// Epilogues:  f32     y = acc * scale
//             resid   y += acc * scale           (x + attn / x + ff, residual kept in f32)
//             gelu    y = bf16(gelu(acc*scale))   (linear1 + activation)
//             qkv     columns [q | k | v] (transformer.rs:197-211): q and k turned by RoPE at
//                     the row's position (rope.rs:81-95), q kept f32, k and v written into
//                     the cache slot of the row's stream (complete_kv, transformer.rs:84-91),
//                     a KV head repeated over the query heads that share it.
//
// Tensor-core mapping (mma.m16n8k16 bf16, f32 accumulate). Within each 16-wide k block the MMA's
// k slots are bound to memory so that every thread's B operand is 4 consecutive int8 weights
// (one 32-bit shared load, converted in registers) and its A operand is 4 consecutive bf16
// (one 64-bit shared load): slot 2t,2t+1 -> k 4t,4t+1 and slot 2t+8,2t+9 -> k 4t+2,4t+3. A and
// B use the same binding, so the dot product is unchanged.
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int BM = 64, BN = 64, BK = 64;
constexpr int kThreads = 128;
constexpr int kStages = 3;
constexpr int kAStride = BK * 2 + 32;  // bytes per A row of a stage (160: conflict-free 8B loads)
constexpr int kBStride = BK + 16;      // bytes per int8 B row (80: conflict-free 4B loads)
constexpr int kAStageBytes = BM * kAStride;
constexpr int kBStageBytes = BN * kBStride;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const int n = valid ? 16 : 0;  // zero-fill rows past M
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)),
                 "l"(gmem), "r"(n)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t i8x2_to_bf16x2(uint32_t w, int shift) {
    const float lo = (float)(int8_t)(w >> shift);
    const float hi = (float)(int8_t)(w >> (shift + 8));
    return pack_bf16x2(lo, hi);
}

__device__ __forceinline__ void mma_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float gelu(float x, int tanh_form) {
    if (tanh_form) {
        const float u2 = (x * x * 0.07135482f + 1.595769f) * x;
        return x / (1.0f + expf(-u2));
    }
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

// One k-tile (BK) of the warp's 32x32 block: a_base/a_stride address A rows (k offset applied
// by the caller), b_tile is the int8 stage.
__device__ __forceinline__ void mma_tile(float (&acc)[2][4][4], const unsigned char* a_base,
                                         int a_stride, const unsigned char* b_tile, int wm, int wn,
                                         int g, int t) {
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
        uint32_t af[2][4];
#pragma unroll
        for (int mi = 0; mi < 2; ++mi) {
            const int r = wm * 32 + mi * 16 + g;
            const uint2 lo = *reinterpret_cast<const uint2*>(a_base + r * a_stride + kk * 32 + t * 8);
            const uint2 hi =
                *reinterpret_cast<const uint2*>(a_base + (r + 8) * a_stride + kk * 32 + t * 8);
            af[mi][0] = lo.x;
            af[mi][1] = hi.x;
            af[mi][2] = lo.y;
            af[mi][3] = hi.y;
        }
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) {
            const int n = wn * 32 + ni * 8 + g;
            const uint32_t wq = *reinterpret_cast<const uint32_t*>(b_tile + n * kBStride + kk * 16 + t * 4);
            const uint32_t b0 = i8x2_to_bf16x2(wq, 0), b1 = i8x2_to_bf16x2(wq, 16);
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) mma_bf16(acc[mi][ni], af[mi], b0, b1);
        }
    }
}

__device__ __forceinline__ void rot(float& x0, float& x1, int pos, float inv_freq) {
    float sn, cs;
    sincosf((float)pos * inv_freq, &sn, &cs);
    const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    x0 = y0;
    x1 = y1;
}

// Epilogue for one pair of adjacent output columns (n even) of row m.
template <int EPI>
__device__ __forceinline__ void epilogue_pair(const LinearArgs& p, int m, int n, float c0,
                                              float c1) {
    const float v0 = c0 * p.scale[n], v1 = c1 * p.scale[n + 1];
    const long long at = (long long)m * p.N + n;
    if (EPI == EPI_F32) {
        *reinterpret_cast<float2*>(p.y + at) = make_float2(v0, v1);
    } else if (EPI == EPI_RESID) {
        float2* y = reinterpret_cast<float2*>(p.y + at);
        const float2 o = *y;
        *y = make_float2(o.x + v0, o.y + v1);
    } else if (EPI == EPI_GELU) {
        *reinterpret_cast<uint32_t*>(p.yb + at) =
            pack_bf16x2(gelu(v0, p.gelu_tanh), gelu(v1, p.gelu_tanh));
    } else {  // EPI_QKV
        const int hd = p.heads * kHeadDim, kvd = p.kv_heads * kHeadDim;
        const int sid = p.row_stream[m], pos = p.row_pos[m];
        const int d = n % kHeadDim;
        float x0 = v0, x1 = v1;
        if (n < hd) {
            rot(x0, x1, pos, p.inv_freq[d >> 1]);
            *reinterpret_cast<float2*>(p.yq + (long long)m * hd + n) = make_float2(x0, x1);
            return;
        }
        if (sid < 0 || sid >= p.num_streams || pos < 0 || pos >= p.capacity) {
            set_error(p.err, DEV_ERR_CAPACITY);
            return;
        }
        const bool is_k = n < hd + kvd;
        const int kvh = (n - hd - (is_k ? 0 : kvd)) / kHeadDim;
        if (is_k) rot(x0, x1, pos, p.inv_freq[d >> 1]);
        const uint32_t packed = pack_bf16x2(x0, x1);
        const int group = p.heads / p.kv_heads;
        __nv_bfloat16* base = (is_k ? p.k_cache : p.v_cache) +
                              ((long long)sid * p.capacity + pos) * hd + d;
        for (int rep = 0; rep < group; ++rep)
            *reinterpret_cast<uint32_t*>(base + (kvh * group + rep) * kHeadDim) = packed;
    }
}

template <bool LN, int EPI>
__global__ void __launch_bounds__(kThreads) linear_kernel(LinearArgs p) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int wm = warp >> 1, wn = warp & 1;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int KT = p.K / BK;
    const int a_res_stride = p.K * 2 + 32;  // resident LN tile
    unsigned char* a_smem = smem;
    unsigned char* b_smem = smem + (LN ? BM * a_res_stride : kStages * kAStageBytes);

    auto load_b = [&](int kt, int st) {
        unsigned char* dst = b_smem + st * kBStageBytes;
#pragma unroll
        for (int i = 0; i < (BN * BK / 16) / kThreads; ++i) {
            const int c = tid + i * kThreads;
            const int r = c >> 2, col = (c & 3) * 16;
            cp_async16(dst + r * kBStride + col, p.w + (long long)(n0 + r) * p.K + kt * BK + col, true);
        }
    };
    auto load_a = [&](int kt, int st) {
        unsigned char* dst = a_smem + st * kAStageBytes;
#pragma unroll
        for (int i = 0; i < (BM * BK * 2 / 16) / kThreads; ++i) {
            const int c = tid + i * kThreads;
            const int r = c >> 3, col = (c & 7) * 16;
            const int gm = m0 + r;
            const bool valid = gm < p.M;
            const unsigned char* src = reinterpret_cast<const unsigned char*>(
                p.a + (long long)(valid ? gm : 0) * p.K + kt * BK) + col;
            cp_async16(dst + r * kAStride + col, src, valid);
        }
    };

    // Start the weight stream first; the LN prologue overlaps it.
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < KT) {
            if (!LN) load_a(s, s);
            load_b(s, s);
        }
        cp_async_commit();
    }

    if (LN) {
        // LayerNorm of this CTA's BM rows into the resident bf16 tile.
        for (int r = warp; r < BM; r += kThreads / 32) {
            const int gm = m0 + r;
            unsigned char* dst = a_smem + r * a_res_stride;
            if (gm >= p.M) {
                for (int k = lane * 4; k < p.K; k += 128)
                    *reinterpret_cast<uint2*>(dst + k * 2) = make_uint2(0, 0);
                continue;
            }
            const float* xr = p.x + (long long)gm * p.K;
            float xv[32];
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int k = lane * 4 + i * 128;
                if (k < p.K) {
                    const float4 v = *reinterpret_cast<const float4*>(xr + k);
                    xv[4 * i] = v.x; xv[4 * i + 1] = v.y; xv[4 * i + 2] = v.z; xv[4 * i + 3] = v.w;
                    sum += (v.x + v.y) + (v.z + v.w);
                }
            }
            const float mean = warp_sum(sum) / (float)p.K;
            float var = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int k = lane * 4 + i * 128;
                if (k < p.K) {
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float c = xv[4 * i + e] - mean;
                        var = fmaf(c, c, var);
                    }
                }
            }
            const float inv = 1.0f / sqrtf(warp_sum(var) / (float)p.K + 1e-5f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int k = lane * 4 + i * 128;
                if (k < p.K) {
                    const float4 gm4 = *reinterpret_cast<const float4*>(p.ln_g + k);
                    const float4 bt4 = *reinterpret_cast<const float4*>(p.ln_b + k);
                    const float y0 = (xv[4 * i] - mean) * inv * gm4.x + bt4.x;
                    const float y1 = (xv[4 * i + 1] - mean) * inv * gm4.y + bt4.y;
                    const float y2 = (xv[4 * i + 2] - mean) * inv * gm4.z + bt4.z;
                    const float y3 = (xv[4 * i + 3] - mean) * inv * gm4.w + bt4.w;
                    *reinterpret_cast<uint2*>(dst + k * 2) = make_uint2(pack_bf16x2(y0, y1), pack_bf16x2(y2, y3));
                }
            }
        }
        __syncthreads();
    }

    float acc[2][4][4];
#pragma unroll
    for (int mi = 0; mi < 2; ++mi)
#pragma unroll
        for (int ni = 0; ni < 4; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mi][ni][e] = 0.f;

    for (int kt = 0; kt < KT; ++kt) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        const int nxt = kt + kStages - 1;
        if (nxt < KT) {
            if (!LN) load_a(nxt, nxt % kStages);
            load_b(nxt, nxt % kStages);
        }
        cp_async_commit();
        const int st = kt % kStages;
        if (LN)
            mma_tile(acc, a_smem + kt * BK * 2, a_res_stride, b_smem + st * kBStageBytes, wm, wn, g, t);
        else
            mma_tile(acc, a_smem + st * kAStageBytes, kAStride, b_smem + st * kBStageBytes, wm, wn, g, t);
    }
    cp_async_wait<0>();

#pragma unroll
    for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
        for (int ni = 0; ni < 4; ++ni) {
            const int m = m0 + wm * 32 + mi * 16 + g;
            const int n = n0 + wn * 32 + ni * 8 + 2 * t;
            if (m < p.M) epilogue_pair<EPI>(p, m, n, acc[mi][ni][0], acc[mi][ni][1]);
            if (m + 8 < p.M) epilogue_pair<EPI>(p, m + 8, n, acc[mi][ni][2], acc[mi][ni][3]);
        }
    }
}

template <bool LN, int EPI>
void launch_typed(const LinearArgs& a, cudaStream_t s) {
    const size_t smem = (LN ? (size_t)BM * (a.K * 2 + 32) : (size_t)kStages * kAStageBytes) +
                        (size_t)kStages * kBStageBytes;
    cudaFuncSetAttribute(linear_kernel<LN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    dim3 grid(a.N / BN, (a.M + BM - 1) / BM);
    linear_kernel<LN, EPI><<<grid, kThreads, smem, s>>>(a);
}

}  // namespace

void launch_linear(const LinearArgs& a, bool ln, LinearEpi epi, cudaStream_t s) {
    if (ln) {
        switch (epi) {
            case EPI_F32: launch_typed<true, EPI_F32>(a, s); break;
            case EPI_QKV: launch_typed<true, EPI_QKV>(a, s); break;
            case EPI_RESID: launch_typed<true, EPI_RESID>(a, s); break;
            case EPI_GELU: launch_typed<true, EPI_GELU>(a, s); break;
        }
    } else {
        switch (epi) {
            case EPI_F32: launch_typed<false, EPI_F32>(a, s); break;
            case EPI_QKV: launch_typed<false, EPI_QKV>(a, s); break;
            case EPI_RESID: launch_typed<false, EPI_RESID>(a, s); break;
            case EPI_GELU: launch_typed<false, EPI_GELU>(a, s); break;
        }
    }
}

}  // namespace ptts
