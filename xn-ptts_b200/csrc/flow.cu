// Flow head kernels (sm_100a): the per-row pieces of FlowLM's frame tail around the flow net's
// tensor-core linears (linear_tc.cu, EPI_BIAS / EPI_COND / EPI_BIAS_SILU / EPI_GATE_RESID).
//   flow_small_kernel     y = a W^T + b (+ add) for K <= 64 (input_linear, input_proj), f32 math
//   flow_norm_eos_kernel  out_norm LayerNorm (eps 1e-5) -> bf16 hi/lo rows and the EOS logit
//   flow_ln_mod_kernel    LayerNorm (eps 1e-6, affine or not) then modulate, x (1 + scale) + shift
//   flow_out_kernel       final linear (ldim outputs) and the solver update cur + step * dir
// All LayerNorms use the biased variance (transformer.rs:547-548, mlp.rs:97-99 via xn's
// LayerNorm), mean and variance in two passes, as ln_kernel does.
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int kSmallRows = 16;

__global__ void __launch_bounds__(128) flow_small_kernel(FlowSmallArgs p) {
    extern __shared__ float sa[];  // [kSmallRows][K]
    grid_dep_wait();
    grid_dep_launch();
    const int m0 = blockIdx.y * kSmallRows, n = blockIdx.x * 128 + threadIdx.x;
    for (int i = threadIdx.x; i < kSmallRows * p.K; i += 128) {
        const int r = i / p.K, k = i - r * p.K, m = m0 + r;
        sa[i] = m < p.M ? (p.a ? p.a[(long long)m * p.K + k] : p.a_row[k]) : 0.f;
    }
    __syncthreads();
    if (n >= p.N) return;
    float acc[kSmallRows];
#pragma unroll
    for (int r = 0; r < kSmallRows; ++r) acc[r] = 0.f;
    for (int k = 0; k < p.K; ++k) {
        const float wk = __ldg(p.w + (long long)n * p.K + k);
#pragma unroll
        for (int r = 0; r < kSmallRows; ++r) acc[r] = fmaf(sa[r * p.K + k], wk, acc[r]);
    }
    const float b = p.bias ? p.bias[n] : 0.f, add = p.add ? p.add[n] : 0.f;
#pragma unroll
    for (int r = 0; r < kSmallRows; ++r) {
        const int m = m0 + r;
        if (m >= p.M) break;
        const float v = acc[r] + b + add;
        if (p.yb) p.yb[(long long)m * p.N + n] = __float2bfloat16_rn(v);
        else p.y[(long long)m * p.N + n] = v;
    }
}

// Mean and 1/sqrt(var + eps) of a row held as PER floats per lane.
template <int PER>
__device__ __forceinline__ void row_stats(const float (&v)[PER], int d, float eps, float& mean, float& inv) {
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) sum += v[i];
    mean = warp_sum(sum) / (float)d;
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const float c = v[i] - mean;
        var = fmaf(c, c, var);
    }
    inv = 1.0f / sqrtf(warp_sum(var) / (float)d + eps);
}

__device__ __forceinline__ void store_bf16_hilo(__nv_bfloat16* hi, __nv_bfloat16* lo, long long at, float a,
                                                float b, float c, float d) {
    uint2 h, l;
    h.x = pack_bf16x2(a, b);
    h.y = pack_bf16x2(c, d);
    l.x = pack_bf16x2(a - bf16lo(h.x), b - bf16hi(h.x));
    l.y = pack_bf16x2(c - bf16lo(h.y), d - bf16hi(h.y));
    *reinterpret_cast<uint2*>(hi + at) = h;
    *reinterpret_cast<uint2*>(lo + at) = l;
}

// One warp per row; lane owns the float4 quads lane + 32 i.
template <int PER>
__global__ void __launch_bounds__(128) flow_norm_eos_kernel(FlowNormArgs p) {
    grid_dep_wait();
    grid_dep_launch();
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= p.M) return;
    constexpr int d = PER * 32, Q = PER / 4;
    float v[PER];
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        const float4 x = *reinterpret_cast<const float4*>(p.x + (long long)row * d + 4 * (lane + 32 * i));
        v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
    }
    if (p.gamma) {
        float mean, inv;
        row_stats<PER>(v, d, p.eps, mean, inv);
#pragma unroll
        for (int i = 0; i < Q; ++i) {
            const int k = 4 * (lane + 32 * i);
            const float4 g = *reinterpret_cast<const float4*>(p.gamma + k);
            const float4 b = *reinterpret_cast<const float4*>(p.beta + k);
            v[4 * i] = (v[4 * i] - mean) * inv * g.x + b.x;
            v[4 * i + 1] = (v[4 * i + 1] - mean) * inv * g.y + b.y;
            v[4 * i + 2] = (v[4 * i + 2] - mean) * inv * g.z + b.z;
            v[4 * i + 3] = (v[4 * i + 3] - mean) * inv * g.w + b.w;
        }
    }
    float e = 0.f;
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        const int k = 4 * (lane + 32 * i);
        const float4 w = *reinterpret_cast<const float4*>(p.eos_w + k);
        e = fmaf(v[4 * i], w.x, e);
        e = fmaf(v[4 * i + 1], w.y, e);
        e = fmaf(v[4 * i + 2], w.z, e);
        e = fmaf(v[4 * i + 3], w.w, e);
        store_bf16_hilo(p.hi, p.lo, (long long)row * d + k, v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    }
    e = warp_sum(e);
    if (lane == 0) p.eos[row] = e + p.eos_b;
}

template <int PER>
__global__ void __launch_bounds__(128) flow_ln_mod_kernel(FlowModArgs p) {
    grid_dep_wait();
    grid_dep_launch();
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= p.M) return;
    constexpr int C = PER * 32, Q = PER / 4;
    float v[PER];
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        const float4 x = *reinterpret_cast<const float4*>(p.x + (long long)row * C + 4 * (lane + 32 * i));
        v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
    }
    float mean, inv;
    row_stats<PER>(v, C, p.eps, mean, inv);
    const float* sh = p.shift + (long long)row * p.stride;
    const float* sc = p.scale + (long long)row * p.stride;
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        const int k = 4 * (lane + 32 * i);
        float4 g = make_float4(1.f, 1.f, 1.f, 1.f), b = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.gamma) {
            g = *reinterpret_cast<const float4*>(p.gamma + k);
            b = *reinterpret_cast<const float4*>(p.beta + k);
        }
        const float4 s = *reinterpret_cast<const float4*>(sc + k);
        const float4 t = *reinterpret_cast<const float4*>(sh + k);
        const float y0 = ((v[4 * i] - mean) * inv * g.x + b.x) * (1.f + s.x) + t.x;
        const float y1 = ((v[4 * i + 1] - mean) * inv * g.y + b.y) * (1.f + s.y) + t.y;
        const float y2 = ((v[4 * i + 2] - mean) * inv * g.z + b.z) * (1.f + s.z) + t.z;
        const float y3 = ((v[4 * i + 3] - mean) * inv * g.w + b.w) * (1.f + s.w) + t.w;
        if (p.y) *reinterpret_cast<float4*>(p.y + (long long)row * C + k) = make_float4(y0, y1, y2, y3);
        else store_bf16_hilo(p.hi, p.lo, (long long)row * C + k, y0, y1, y2, y3);
    }
}

// The flow net's last two steps in one pass, one warp per row (FinalLayer, mlp.rs:125-157, and
// the solver update): LayerNorm (no affine) + modulate as flow_ln_mod_kernel does, then the L
// (<= 32) outputs h . w[j] + bias[j] and out = cur + step_scale * dir. Each lane sums its 16
// columns for every output; a reduce-scatter over the warp (31 shuffles) leaves output j's sum
// in lane j. The modulated row never goes to memory.
template <int PER>
__global__ void __launch_bounds__(128) flow_final_kernel(FlowModArgs m, FlowOutArgs o) {
    grid_dep_wait();
    grid_dep_launch();
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= m.M) return;
    constexpr int C = PER * 32, Q = PER / 4;
    float v[PER];
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        const float4 x = *reinterpret_cast<const float4*>(m.x + (long long)row * C + 4 * (lane + 32 * i));
        v[4 * i] = x.x; v[4 * i + 1] = x.y; v[4 * i + 2] = x.z; v[4 * i + 3] = x.w;
    }
    float mean, inv;
    row_stats<PER>(v, C, m.eps, mean, inv);
    const float* sh = m.shift + (long long)row * m.stride;
    const float* sc = m.scale + (long long)row * m.stride;
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        const int k = 4 * (lane + 32 * i);
        const float4 sv = *reinterpret_cast<const float4*>(sc + k);
        const float4 t = *reinterpret_cast<const float4*>(sh + k);
        v[4 * i] = (v[4 * i] - mean) * inv * (1.f + sv.x) + t.x;
        v[4 * i + 1] = (v[4 * i + 1] - mean) * inv * (1.f + sv.y) + t.y;
        v[4 * i + 2] = (v[4 * i + 2] - mean) * inv * (1.f + sv.z) + t.z;
        v[4 * i + 3] = (v[4 * i + 3] - mean) * inv * (1.f + sv.w) + t.w;
    }
    float part[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        float a = 0.f;
        if (j < o.L) {
            const float* wr = o.w + (long long)j * C;
#pragma unroll
            for (int i = 0; i < Q; ++i) {
                const float4 w = __ldg(reinterpret_cast<const float4*>(wr + 4 * (lane + 32 * i)));
                a = fmaf(v[4 * i], w.x, a);
                a = fmaf(v[4 * i + 1], w.y, a);
                a = fmaf(v[4 * i + 2], w.z, a);
                a = fmaf(v[4 * i + 3], w.w, a);
            }
        }
        part[j] = a;
    }
    // Reduce-scatter: after the stage of offset `off` a lane holds `off` sums, those of the
    // outputs whose bits above `off` match its own lane bits; at the end part[0] is output lane.
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int j = 0; j < off; ++j) {
            const float send = upper ? part[j] : part[j + off];
            const float keep = upper ? part[j + off] : part[j];
            part[j] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
    }
    if (lane < o.L) {
        const float dir = part[0] + o.bias[lane];
        const long long at = (long long)row * o.L + lane;
        o.out[at] = o.cur ? o.cur[at] + o.step_scale * dir : dir;
    }
}

// Eight rows per block (one per warp); the weights sit transposed in shared memory, [C][L + 1]
// (the extra column keeps both the transposing stores and the reads free of bank conflicts),
// so lane j reads output j's column. L <= 64 (lanes j and j + 32).
__global__ void __launch_bounds__(256) flow_out_kernel(FlowOutArgs p) {
    extern __shared__ float wt[];  // [C][L + 1]
    const int ld = p.L + 1;
    grid_dep_wait();
    grid_dep_launch();
    {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int j = warp; j < p.L; j += blockDim.x >> 5)   // w[j][k]: coalesced along k
            for (int k = lane; k < p.C; k += 32) wt[k * ld + j] = __ldg(p.w + (long long)j * p.C + k);
    }
    __syncthreads();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= p.M) return;
    const float* h = p.h + (long long)row * p.C;
    const int j0 = lane < p.L ? lane : 0, j1 = lane + 32 < p.L ? lane + 32 : 0;  // in-row columns
    float a0 = 0.f, a1 = 0.f;
    for (int k0 = 0; k0 < p.C; k0 += 32) {
        const float hv = h[k0 + lane];
#pragma unroll 8
        for (int i = 0; i < 32; ++i) {
            const float hk = __shfl_sync(0xffffffffu, hv, i);
            const float* wr = wt + (k0 + i) * ld;
            a0 = fmaf(hk, wr[j0], a0);
            if (p.L > 32) a1 = fmaf(hk, wr[j1], a1);
        }
    }
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        const int j = lane + 32 * h2;
        if (j >= p.L) break;
        const float dir = (h2 ? a1 : a0) + p.bias[j];
        const long long at = (long long)row * p.L + j;
        p.out[at] = p.cur ? p.cur[at] + p.step_scale * dir : dir;
    }
}

}  // namespace

void launch_flow_small(const FlowSmallArgs& a, cudaStream_t s) {
    const dim3 grid((a.N + 127) / 128, (a.M + kSmallRows - 1) / kSmallRows);
    launch_k(flow_small_kernel, grid, dim3(128), sizeof(float) * kSmallRows * a.K, s, a);
}

void launch_flow_norm_eos(const FlowNormArgs& a, cudaStream_t s) {
    const dim3 grid((a.M + 3) / 4);
    switch (a.d) {
        case 128: launch_k(flow_norm_eos_kernel<4>, grid, dim3(128), 0, s, a); break;
        case 256: launch_k(flow_norm_eos_kernel<8>, grid, dim3(128), 0, s, a); break;
        case 512: launch_k(flow_norm_eos_kernel<16>, grid, dim3(128), 0, s, a); break;
        case 1024: launch_k(flow_norm_eos_kernel<32>, grid, dim3(128), 0, s, a); break;
        default: break;  // refused at flow creation
    }
}

void launch_flow_ln_mod(const FlowModArgs& a, cudaStream_t s) {
    const dim3 grid((a.M + 3) / 4);
    switch (a.C) {
        case 128: launch_k(flow_ln_mod_kernel<4>, grid, dim3(128), 0, s, a); break;
        case 256: launch_k(flow_ln_mod_kernel<8>, grid, dim3(128), 0, s, a); break;
        case 512: launch_k(flow_ln_mod_kernel<16>, grid, dim3(128), 0, s, a); break;
        case 1024: launch_k(flow_ln_mod_kernel<32>, grid, dim3(128), 0, s, a); break;
        default: break;  // refused at flow creation
    }
}

bool launch_flow_final(const FlowModArgs& m, const FlowOutArgs& o, cudaStream_t s) {
    if (m.C != 512 || o.C != 512 || o.L > 32 || m.gamma || m.y || m.hi) return false;
    launch_k(flow_final_kernel<16>, dim3((m.M + 3) / 4), dim3(128), 0, s, m, o);
    return true;
}

void launch_flow_out(const FlowOutArgs& a, cudaStream_t s) {
    const size_t smem = sizeof(float) * a.C * (a.L + 1);
    set_max_dynamic_smem(reinterpret_cast<const void*>(flow_out_kernel), 200 * 1024);
    launch_k(flow_out_kernel, dim3((a.M + 7) / 8), dim3(256), smem, s, a);
}

}  // namespace ptts
