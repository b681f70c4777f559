// int8-weight linears of the flow-LM layer with their neighbours fused in.
//
// Reference: Q::LinearQ::forward for in_proj, out_proj, linear1 and linear2
// (ptts/src/transformer.rs:195, :224, :627), GELU (:620-625) and the residual adds (:616, :634).
// Weights are int8 [out][in] with one f32 scale per output row, so
// y[m][n] = scale[n] * sum_k a[m][k] * q[n][k]. int8 values are exact in bf16, so the products
// run on the tensor cores and the scale is applied once in the epilogue.
//
// Activations. Every A operand of the layer stack arrives as two f16 planes, hi = f16(a) and
// lo = f16(a - hi) (saturating at +-65504), and each tile runs two MMAs (hi and lo) into one f32
// accumulator: about 22 mantissa bits of the f32 activation reach the product, so the GEMMs are
// f32-grade. (With the bf16 KV cache the only rounding to 16-bit storage, two implementations of
// the stack agree to ~1e-3 instead of parting by ~1e-3 per layer, as rounding GEMM inputs to
// bf16 makes them.) int8 weights convert to f16 exactly with a byte permute and one packed
// subtract. The plain linear op (ptts_b200_linear_i8) takes one bf16 plane and runs on bf16.
//
// Epilogues:  f32      y = acc * scale                 (the plain linear op, one A plane)
//             partial  part[z] = acc * scale           (split-K slice z; summed into the
//                                                      residual by the next LayerNorm kernel)
//             resid    y += acc * scale                (residual update when not split)
//             gelu     ff = gelu(acc * scale) as hi/lo planes (linear1 + activation)
//             qkv      columns [q | k | v] (transformer.rs:197-211): q and k turned by RoPE at
//                      the row's position (rope.rs:81-95), q kept f32, k and v written as bf16
//                      into the cache slot of the row's stream (complete_kv,
//                      transformer.rs:84-91), a KV head repeated over the query heads sharing it.
//
// Tensor-core mapping (mma.m16n8k16 bf16, f32 accumulate). Within each 16-wide k block the MMA's
// k slots are bound to memory so that every thread's B operand is 4 consecutive int8 weights
// (one 32-bit shared load, converted in registers) and its A operand 4 consecutive bf16 (one
// 64-bit shared load): slot 2t,2t+1 -> k 4t,4t+1 and slot 2t+8,2t+9 -> k 4t+2,4t+3. A and B use
// the same binding, so the dot product is unchanged.
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

// Tiles: TM (64, or 32 below 1024 rows so decode sizes fill the GPU) x BN 64 x BK 64, four
// warps: 2 x 2 warp tiles of 32 x 32 (TM 64) or 1 x 4 of 32 x 16 (TM 32).
constexpr int BN = 64, BK = 64;
constexpr int kThreads = 128;
constexpr int kAStride = BK * 2 + 32;  // bytes per A row of a stage (160: conflict-free 8B loads)
constexpr int kBStride = BK + 16;      // bytes per int8 B row (80: conflict-free 4B loads)
constexpr int kBStageBytes = BN * kBStride;
template <int TM>
struct Tile {
    // Three stages: deeper rings (6 / 4) measured slower, as they cost CTAs per SM.
    static constexpr int kStages = 3;
    static constexpr int kAStageBytes = TM * kAStride;
    static constexpr int kStageBytes = 2 * kAStageBytes + kBStageBytes;  // A hi, A lo, B
    static constexpr int kSmemBytes = kStages * kStageBytes;
    static constexpr int NI = TM == 64 ? 4 : 2;  // 8-column fragments per warp
};

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


// D += A B, m16n8k16, f32 accumulate; A and B both f16 (F16) or both bf16.
template <bool F16>
__device__ __forceinline__ void mma16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    if (F16)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    else
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
    return gelu_erf(x);
}

template <int MI>
__device__ __forceinline__ void load_afrag(uint32_t (&af)[MI][4], const unsigned char* a, int row0,
                                           int kk, int g, int t) {
#pragma unroll
    for (int mi = 0; mi < MI; ++mi) {
        const int r = row0 + mi * 16 + g;
        const uint2 lo = *reinterpret_cast<const uint2*>(a + r * kAStride + kk * 32 + t * 8);
        const uint2 hi = *reinterpret_cast<const uint2*>(a + (r + 8) * kAStride + kk * 32 + t * 8);
        af[mi][0] = lo.x;
        af[mi][1] = hi.x;
        af[mi][2] = lo.y;
        af[mi][3] = hi.y;
    }
}

// One k-tile (BK) of the warp's (16 MI) x (8 NI) block at (row0, col0), with the lo plane when
// present. The hi products of all fragments are issued before the lo ones, so no MMA waits on
// the accumulator of the one just issued.
template <int MI, int NI, bool F16>
__device__ __forceinline__ void mma_tile(float (&acc)[MI][NI][4], const unsigned char* a_hi,
                                         const unsigned char* a_lo, bool has_lo,
                                         const unsigned char* b_tile, int row0, int col0, int g,
                                         int t) {
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
        uint32_t ah[MI][4], al[MI][4], b0[NI], b1[NI];
        load_afrag<MI>(ah, a_hi, row0, kk, g, t);
#pragma unroll
        for (int ni = 0; ni < NI; ++ni) {
            const int n = col0 + ni * 8 + g;
            const uint32_t wq = *reinterpret_cast<const uint32_t*>(b_tile + n * kBStride + kk * 16 + t * 4);
            i8x4_convert<F16>(wq, b0[ni], b1[ni]);
        }
#pragma unroll
        for (int ni = 0; ni < NI; ++ni)
#pragma unroll
            for (int mi = 0; mi < MI; ++mi) mma16<F16>(acc[mi][ni], ah[mi], b0[ni], b1[ni]);
        if (has_lo) {
            load_afrag<MI>(al, a_lo, row0, kk, g, t);
#pragma unroll
            for (int ni = 0; ni < NI; ++ni)
#pragma unroll
                for (int mi = 0; mi < MI; ++mi) mma16<F16>(acc[mi][ni], al[mi], b0[ni], b1[ni]);
        }
    }
}

// RoPE of the pair (x0, x1) by the table entry t = (cos, sin); rope.rs:37-95 rounding order.
__device__ __forceinline__ void rot(float& x0, float& x1, float2 t) {
    const float y0 = __fsub_rn(__fmul_rn(x0, t.x), __fmul_rn(x1, t.y));
    const float y1 = __fadd_rn(__fmul_rn(x0, t.y), __fmul_rn(x1, t.x));
    x0 = y0;
    x1 = y1;
}

// Epilogue for one pair of adjacent output columns (n even) of row m, split slice z.
template <int EPI>
__device__ __forceinline__ void epilogue_pair(const LinearArgs& p, int m, int n, int z, float c0,
                                              float c1) {
    const float v0 = c0 * p.scale[n], v1 = c1 * p.scale[n + 1];
    const long long at = (long long)m * p.N + n;
    if (EPI == EPI_F32) {
        *reinterpret_cast<float2*>(p.y + at) = make_float2(v0, v1);
    } else if (EPI == EPI_PARTIAL) {
        *reinterpret_cast<float2*>(p.y + (long long)z * p.M * p.N + at) = make_float2(v0, v1);
    } else if (EPI == EPI_RESID) {
        float2* y = reinterpret_cast<float2*>(p.y + at);
        const float2 o = *y;
        *y = make_float2(o.x + v0, o.y + v1);
    } else if (EPI == EPI_GELU) {
        uint32_t hi, lo;
        split_f16x2(gelu(v0, p.gelu_tanh), gelu(v1, p.gelu_tanh), hi, lo);
        static_cast<uint32_t*>(p.yb)[at >> 1] = hi;
        static_cast<uint32_t*>(p.yb_lo)[at >> 1] = lo;
    }
}

// EPI_QKV for the column pair (n, n+1) of row m at (sid, pos), with its RoPE table entry t
// (loaded by the caller before any store, so no load waits behind the stores).
__device__ __forceinline__ void qkv_pair(const LinearArgs& p, int m, int n, float c0, float c1, int sid,
                                         int pos, float2 t) {
    // `pos` is the row's cache slot here (the RoPE factors t come from its position).
    const int hd = p.heads * kHeadDim, kvd = p.kv_heads * kHeadDim;
    const int d = n % kHeadDim;
    float x0 = c0 * p.scale[n], x1 = c1 * p.scale[n + 1];
    if (n < hd) {
        rot(x0, x1, t);
        if (p.yq_hi) {
            x0 *= p.yq_scale;
            x1 *= p.yq_scale;
            const uint32_t hi = pack_bf16x2(x0, x1);
            *reinterpret_cast<uint32_t*>(p.yq_hi + (long long)m * hd + n) = hi;
            *reinterpret_cast<uint32_t*>(p.yq_lo + (long long)m * hd + n) = pack_bf16x2(x0 - bf16lo(hi), x1 - bf16hi(hi));
        } else {
            *reinterpret_cast<float2*>(p.yq + (long long)m * hd + n) = make_float2(x0, x1);
        }
        return;
    }
    if (sid < 0 || sid >= p.num_streams || pos < 0 || pos >= p.capacity) {
        set_error(p.err, DEV_ERR_CAPACITY);
        return;
    }
    const bool is_k = n < hd + kvd;
    const int kvh = (n - hd - (is_k ? 0 : kvd)) / kHeadDim;
    if (is_k) rot(x0, x1, t);
    const uint32_t packed = pack_bf16x2(x0, x1);
    const int group = p.heads / p.kv_heads;
    __nv_bfloat16* cache = is_k ? p.k_cache : p.v_cache;
    for (int rep = 0; rep < group; ++rep)
        *reinterpret_cast<uint32_t*>(cache + kv_offset(sid, pos, kvh * group + rep, p.num_streams, p.capacity) + d) =
            packed;
}

template <int EPI, int TM, bool F16>
__global__ void __launch_bounds__(kThreads) linear_kernel(LinearArgs p) {
    using T = Tile<TM>;
    constexpr int MI = 2, NI = T::NI;
    constexpr int kStages = T::kStages;
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int row0 = TM == 64 ? (warp >> 1) * 32 : 0;
    const int col0 = TM == 64 ? (warp & 1) * 32 : warp * 16;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * TM, z = blockIdx.z;
    const int k_len = p.K / p.splits;
    const int k0 = z * k_len;
    const int KT = k_len / BK;
    const bool has_lo = p.a_lo != nullptr;

    auto load_b = [&](int kt, int st) {
        unsigned char* bdst = smem + st * T::kStageBytes + 2 * T::kAStageBytes;
        const int kb = k0 + kt * BK;
#pragma unroll
        for (int i = 0; i < (BN * BK / 16) / kThreads; ++i) {
            const int c = tid + i * kThreads;
            const int r = c >> 2, col = (c & 3) * 16;
            cp_async16(bdst + r * kBStride + col, p.w + (long long)(n0 + r) * p.K + kb + col, true);
        }
    };
    auto load_a = [&](int kt, int st) {
        unsigned char* base = smem + st * T::kStageBytes;
        const int kb = k0 + kt * BK;
#pragma unroll
        for (int i = 0; i < (TM * BK * 2 / 16) / kThreads; ++i) {
            const int c = tid + i * kThreads;
            const int r = c >> 3, col = (c & 7) * 16;
            const int gm = m0 + r;
            const bool valid = gm < p.M;
            const long long off = 2 * ((long long)(valid ? gm : 0) * p.K + kb);  // bytes
            cp_async16(base + r * kAStride + col,
                       static_cast<const unsigned char*>(p.a) + off + col, valid);
            if (has_lo)
                cp_async16(base + T::kAStageBytes + r * kAStride + col,
                           static_cast<const unsigned char*>(p.a_lo) + off + col, valid);
        }
    };

    // The weights never change, so their first stages load before the wait on the kernel that
    // produced A; the first commit group then holds them too.
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s)
        if (s < KT) load_b(s, s);
    grid_dep_wait();
    grid_dep_launch();
#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
        if (s < KT) load_a(s, s);
        cp_async_commit();
    }

    float acc[MI][NI][4];
#pragma unroll
    for (int mi = 0; mi < MI; ++mi)
#pragma unroll
        for (int ni = 0; ni < NI; ++ni)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mi][ni][e] = 0.f;

    for (int kt = 0; kt < KT; ++kt) {
        cp_async_wait<kStages - 2>();
        __syncthreads();
        const int nxt = kt + kStages - 1;
        if (nxt < KT) {
            load_a(nxt, nxt % kStages);
            load_b(nxt, nxt % kStages);
        }
        cp_async_commit();
        const unsigned char* base = smem + (kt % kStages) * T::kStageBytes;
        mma_tile<MI, NI, F16>(acc, base, base + T::kAStageBytes, has_lo, base + 2 * T::kAStageBytes,
                              row0, col0, g, t);
    }
    cp_async_wait<0>();

    if constexpr (EPI == EPI_QKV) {
        // Row metadata and RoPE entries of all this thread's outputs first, then the stores.
        int sid[MI][2], pos[MI][2];
        float2 rt[MI][2][NI];
        const bool rotated = n0 < (p.heads + p.kv_heads) * kHeadDim;  // q or k columns (BN | 64)
#pragma unroll
        for (int mi = 0; mi < MI; ++mi)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int m = m0 + row0 + mi * 16 + g + 8 * h;
                sid[mi][h] = m < p.M ? p.row_stream[m] : 0;
                const int rpos = m < p.M ? p.row_pos[m] : 0;
                pos[mi][h] = m < p.M ? p.row_slot[m] : 0;  // cache slot
                const long long trow = (long long)min(max(rpos, 0), p.rope_rows - 1) * kMaxPairs;
#pragma unroll
                for (int ni = 0; ni < NI; ++ni)
                    rt[mi][h][ni] = rotated ? __ldg(p.rope + trow + ((n0 + col0 + ni * 8 + 2 * t) % kHeadDim) / 2)
                                            : make_float2(1.f, 0.f);
            }
#pragma unroll
        for (int mi = 0; mi < MI; ++mi)
#pragma unroll
            for (int ni = 0; ni < NI; ++ni) {
                const int m = m0 + row0 + mi * 16 + g;
                const int n = n0 + col0 + ni * 8 + 2 * t;
                if (m < p.M) qkv_pair(p, m, n, acc[mi][ni][0], acc[mi][ni][1], sid[mi][0], pos[mi][0], rt[mi][0][ni]);
                if (m + 8 < p.M)
                    qkv_pair(p, m + 8, n, acc[mi][ni][2], acc[mi][ni][3], sid[mi][1], pos[mi][1], rt[mi][1][ni]);
            }
    } else {
#pragma unroll
        for (int mi = 0; mi < MI; ++mi) {
#pragma unroll
            for (int ni = 0; ni < NI; ++ni) {
                const int m = m0 + row0 + mi * 16 + g;
                const int n = n0 + col0 + ni * 8 + 2 * t;
                if (m < p.M) epilogue_pair<EPI>(p, m, n, z, acc[mi][ni][0], acc[mi][ni][1]);
                if (m + 8 < p.M) epilogue_pair<EPI>(p, m + 8, n, z, acc[mi][ni][2], acc[mi][ni][3]);
            }
        }
    }
}

// One warp per row: residual (+ split-K partial slices) -> residual, then LayerNorm -> hi/lo.
// transformer.rs:547-548 (eps 1e-5, biased variance); the row sum uses a warp reduction.
// PER = d_model / 32 floats per lane.
template <int PER>
__global__ void __launch_bounds__(128) ln_kernel(LnArgs a) {
    if (threadIdx.x == 0) stamp_mark(a.stamps, a.stamp, STAMP_ENTRY);
    grid_dep_wait();
    if (threadIdx.x == 0) stamp_mark(a.stamps, a.stamp, STAMP_START);
    grid_dep_launch();
    const int row = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= a.M) return;
    constexpr int d = PER * 32;
    constexpr int Q = PER / 4;  // float4 per lane
    float4 x[Q];
    float* xr = a.resid + (long long)row * d;
    // Every load of the row (input, or residual plus up to four split-K slices) is issued
    // before any of them is used.
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        const int k = 4 * (lane + 32 * i);
        if (a.x_bf16) {
            const uint2 u = *reinterpret_cast<const uint2*>(a.x_bf16 + (long long)row * d + k);
            x[i] = make_float4(bf16lo(u.x), bf16hi(u.x), bf16lo(u.y), bf16hi(u.y));
        } else {
            x[i] = *reinterpret_cast<const float4*>(xr + k);
        }
    }
    float4 q[4][Q];
#pragma unroll
    for (int s = 0; s < 4; ++s)
#pragma unroll
        for (int i = 0; i < Q; ++i)
            q[s][i] = s < a.nsplit
                          ? *reinterpret_cast<const float4*>(a.part + ((long long)s * a.M + row) * d + 4 * (lane + 32 * i))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
    float v[PER];
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        float4 y = x[i];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            y.x += q[s][i].x; y.y += q[s][i].y; y.z += q[s][i].z; y.w += q[s][i].w;
        }
        v[4 * i] = y.x; v[4 * i + 1] = y.y; v[4 * i + 2] = y.z; v[4 * i + 3] = y.w;
        if (a.x_bf16 || a.nsplit) *reinterpret_cast<float4*>(xr + 4 * (lane + 32 * i)) = y;
    }
    if (!a.hi) {  // reduce only
        if (lane == 0) stamp_mark(a.stamps, a.stamp, STAMP_END);
        return;
    }
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) sum += v[i];
    const float mean = warp_sum(sum) / (float)d;
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
        const float c = v[i] - mean;
        var = fmaf(c, c, var);
    }
    const float inv = 1.0f / sqrtf(warp_sum(var) / (float)d + 1e-5f);
#pragma unroll
    for (int i = 0; i < Q; ++i) {
        const int k = 4 * (lane + 32 * i);
        const float4 gm = *reinterpret_cast<const float4*>(a.gamma + k);
        const float4 bt = *reinterpret_cast<const float4*>(a.beta + k);
        const float y0 = (v[4 * i] - mean) * inv * gm.x + bt.x;
        const float y1 = (v[4 * i + 1] - mean) * inv * gm.y + bt.y;
        const float y2 = (v[4 * i + 2] - mean) * inv * gm.z + bt.z;
        const float y3 = (v[4 * i + 3] - mean) * inv * gm.w + bt.w;
        uint32_t h01, h23, l01, l23;
        split_f16x2(y0, y1, h01, l01);
        split_f16x2(y2, y3, h23, l23);
        *reinterpret_cast<uint2*>(a.hi + (long long)row * d + k) = make_uint2(h01, h23);
        *reinterpret_cast<uint2*>(a.lo + (long long)row * d + k) = make_uint2(l01, l23);
    }
    if (lane == 0) stamp_mark(a.stamps, a.stamp, STAMP_END);
}

template <int EPI, int TM, bool F16>
void launch_tile(const LinearArgs& a, cudaStream_t s) {
    set_max_dynamic_smem(reinterpret_cast<const void*>(linear_kernel<EPI, TM, F16>), Tile<TM>::kSmemBytes);
    dim3 grid(a.N / BN, (a.M + TM - 1) / TM, a.splits);
    launch_k(linear_kernel<EPI, TM, F16>, grid, dim3(kThreads), Tile<TM>::kSmemBytes, s, a);
}

template <int EPI>
void launch_typed(const LinearArgs& a, cudaStream_t s) {
    if (a.a_f16) {
        if (a.M < 1024) launch_tile<EPI, 32, true>(a, s);
        else launch_tile<EPI, 64, true>(a, s);
    } else {
        if (a.M < 1024) launch_tile<EPI, 32, false>(a, s);
        else launch_tile<EPI, 64, false>(a, s);
    }
}

}  // namespace

bool launch_linear(const LinearArgs& a, LinearEpi epi, cudaStream_t s) {
    // The tcgen05 kernel wherever it applies (decode batches and prompts alike: 56 ms against
    // 90 ms for config 5's 139k-row prefill); weights without an int8 copy (f32 or q8_0
    // layers) only have it. PTTS_B200_GEMM=mma selects the mma.sync kernel where both exist.
    if (a.w == nullptr || a.wblk) return launch_linear_tc(a, epi, s);  // wblk: tcgen05 only
    const char* sel = getenv("PTTS_B200_GEMM");
    const bool use_tc = !(sel && sel[0] == 'm');
    if (use_tc && launch_linear_tc(a, epi, s)) return true;
    launch_linear_mma(a, epi, s);
    return true;
}

void launch_linear_mma(const LinearArgs& a, LinearEpi epi, cudaStream_t s) {
    switch (epi) {
        case EPI_F32: launch_typed<EPI_F32>(a, s); break;
        case EPI_QKV: launch_typed<EPI_QKV>(a, s); break;
        case EPI_RESID: launch_typed<EPI_RESID>(a, s); break;
        case EPI_GELU: launch_typed<EPI_GELU>(a, s); break;
        case EPI_PARTIAL: launch_typed<EPI_PARTIAL>(a, s); break;
    }
}

void launch_ln(const LnArgs& a, cudaStream_t s) {
    const dim3 blocks((a.M + 3) / 4), threads(128);
    switch (a.d) {
        case 128: launch_k(ln_kernel<4>, blocks, threads, 0, s, a); break;
        case 256: launch_k(ln_kernel<8>, blocks, threads, 0, s, a); break;
        case 512: launch_k(ln_kernel<16>, blocks, threads, 0, s, a); break;
        case 1024: launch_k(ln_kernel<32>, blocks, threads, 0, s, a); break;
        default: break;  // refused by the caller (d_model is checked at model creation)
    }
}

}  // namespace ptts
