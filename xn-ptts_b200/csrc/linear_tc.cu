// int8-weight linears on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Same contract as linear.cu (LinearArgs, the five epilogues, A as f16 hi/lo planes or one bf16
// plane, int8 weights with one f32 scale per output row); this file replaces its mma.sync main
// loop.
//
// CTA tile 128 (rows) x 64 (output features), K in steps of 64, a 4-stage shared-memory ring:
//   warps 0-3  loaders: cp.async the A hi and lo planes straight into the 128-byte-swizzled
//              K-major layout the MMA reads (16-byte chunk c of row r lands at chunk c ^ (r & 7)),
//              cp.async the int8 weight tile raw, then convert it in registers to A's type (exact)
//              into the same swizzled layout; fence.proxy.async, then arrive on the stage's
//              `full` barrier. After the main loop they are the epilogue: warp w reads TMEM
//              lanes 32w..32w+31 (one output row per thread) with tcgen05.ld.
//   warp 4     one thread issues tcgen05.mma.cta_group::1.kind::f16 (M=128, N=64, K=16; f16 x
//              f16 or bf16 x bf16 -> f32 in TMEM): per 64-wide K tile 4 steps x (hi, lo), then
//              tcgen05.commit to the stage's `empty` barrier; after the last tile a commit to
//              `done`.
// TMEM: 64 columns (the 128x64 f32 accumulator), allocated and freed by warp 0.
// Every mbarrier wait is bounded and sets DEV_ERR_TIMEOUT; on a timeout the CTA still waits
// (bounded) for its copies and MMAs in flight and frees its TMEM before returning.
// No cluster launch, no multicast.
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int TBM = 128, TBN = 64, TBK = 64;
constexpr int kLoaderWarps = 4;
constexpr int kThreadsTc = (kLoaderWarps + 1) * 32;
constexpr int kStagesTc = 4;
constexpr int kATileBytes = TBM * TBK * 2;   // 16 KB, 128-byte rows
constexpr int kBTileBytes = TBN * TBK * 2;   // 8 KB
constexpr int kBRawBytes = TBN * TBK;        // 4 KB int8
constexpr int kStageTc = 2 * kATileBytes + kBTileBytes + kBRawBytes;  // 44 KB, 1024-aligned
constexpr int kBarOffset = kStagesTc * kStageTc;
constexpr int kSmemTc = 1024 + kBarOffset + 256;  // + alignment slack + barriers/TMEM address
constexpr uint32_t kTmemCols = TBN;

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B both f16 (format 0) or both
// bf16 (format 1, bits 7-9 and 10-12), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdescF16 = (1u << 4) | ((uint32_t)(TBN >> 3) << 17) | ((uint32_t)(TBM >> 4) << 24);
constexpr uint32_t kIdescBf16 = kIdescF16 | (1u << 7) | (1u << 10);

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile at `addr` (1024-aligned):
// start >> 4 in bits 0-13, leading byte offset 1 (unused when swizzled), stride byte offset
// 1024 B (8 rows of 128 B) >> 4 in bits 32-45, version 1 at bit 46, layout SWIZZLE_128B (2) at
// bits 61-63.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 consecutive f32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
          "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
          "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float gelu_tc(float x, int tanh_form) {
    if (tanh_form) {
        const float u2 = (x * x * 0.07135482f + 1.595769f) * x;
        return x / (1.0f + expf(-u2));
    }
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}

__device__ __forceinline__ void rot_tc(float& x0, float& x1, int pos, float inv_freq) {
    float sn, cs;
    sincosf((float)pos * inv_freq, &sn, &cs);
    const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    x0 = y0;
    x1 = y1;
}

// Same arithmetic as linear.cu's epilogue for the column pair (n, n+1) of row m.
template <int EPI>
__device__ __forceinline__ void epi_pair(const LinearArgs& p, int m, int n, int z, float c0, float c1) {
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
        split_f16x2(gelu_tc(v0, p.gelu_tanh), gelu_tc(v1, p.gelu_tanh), hi, lo);
        static_cast<uint32_t*>(p.yb)[at >> 1] = hi;
        static_cast<uint32_t*>(p.yb_lo)[at >> 1] = lo;
    } else {  // EPI_QKV
        const int hd = p.heads * kHeadDim, kvd = p.kv_heads * kHeadDim;
        const int sid = p.row_stream[m], pos = p.row_pos[m];
        const int d = n % kHeadDim;
        float x0 = v0, x1 = v1;
        if (n < hd) {
            rot_tc(x0, x1, pos, p.inv_freq[d >> 1]);
            *reinterpret_cast<float2*>(p.yq + (long long)m * hd + n) = make_float2(x0, x1);
            return;
        }
        if (sid < 0 || sid >= p.num_streams || pos < 0 || pos >= p.capacity) {
            set_error(p.err, DEV_ERR_CAPACITY);
            return;
        }
        const bool is_k = n < hd + kvd;
        const int kvh = (n - hd - (is_k ? 0 : kvd)) / kHeadDim;
        if (is_k) rot_tc(x0, x1, pos, p.inv_freq[d >> 1]);
        const uint32_t packed = pack_bf16x2(x0, x1);
        const int group = p.heads / p.kv_heads;
        __nv_bfloat16* base = (is_k ? p.k_cache : p.v_cache) + ((long long)sid * p.capacity + pos) * hd + d;
        for (int rep = 0; rep < group; ++rep)
            *reinterpret_cast<uint32_t*>(base + (kvh * group + rep) * kHeadDim) = packed;
    }
}

template <int EPI>
__global__ void __launch_bounds__(kThreadsTc, 1) linear_tc_kernel(LinearArgs p) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-aligned for the 128-byte swizzle
    unsigned char* smem = smem_raw + (base - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOffset);
    uint64_t* empty = full + kStagesTc;
    uint64_t* done = empty + kStagesTc;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * TBN, m0 = blockIdx.y * TBM, z = blockIdx.z;
    const int k_len = p.K / p.splits;
    const int k0 = z * k_len;
    const int KT = k_len / TBK;
    const bool has_lo = p.a_lo != nullptr;
    const bool f16 = p.a_f16 != 0;

    if (tid == 0) {
        s_abort = 0;
        for (int s = 0; s < kStagesTc; ++s) {
            mbar_init(&full[s], kLoaderWarps);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    grid_dep_wait();
    grid_dep_launch();

    if (warp < kLoaderWarps) {
        // ---- loaders -------------------------------------------------------------------------
        const int lt = tid;  // 0..127
        bool ok = true;
        // Issue the loads of K tile `it` into its stage.
        auto issue = [&](int it) {
            const int st = it % kStagesTc;
            const uint32_t sa = base + st * kStageTc;
            const int kb = k0 + it * TBK;
            // A: 128 rows x 8 chunks of 16 B per plane; 8 consecutive threads cover one row.
            const int c = lt & 7;
#pragma unroll
            for (int i = 0; i < TBM / 16; ++i) {
                const int r = i * 16 + (lt >> 3);
                const int gm = m0 + r;
                const bool valid = gm < p.M;
                const long long off = 2 * ((long long)(valid ? gm : 0) * p.K + kb + c * 8);  // bytes
                const uint32_t dst = sa + r * 128 + ((c ^ (r & 7)) << 4);
                cp_async16(dst, static_cast<const unsigned char*>(p.a) + off, valid);
                if (has_lo) cp_async16(dst + kATileBytes, static_cast<const unsigned char*>(p.a_lo) + off, valid);
            }
            // B raw: 64 rows x 4 chunks of 16 int8; thread lt takes chunks lt and lt + 128.
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int c = lt + 128 * q;
                const int n = c >> 2, cc = c & 3;
                cp_async16(sa + 2 * kATileBytes + kBTileBytes + n * 64 + cc * 16,
                           p.w + (long long)(n0 + n) * p.K + kb + cc * 16, true);
            }
        };
        // Convert this thread's two raw chunks of K tile `it` into the swizzled f16/bf16 tile.
        auto convert = [&](int it) {
            const int st = it % kStagesTc;
            unsigned char* sp = smem + st * kStageTc;
            const unsigned char* rawb = sp + 2 * kATileBytes + kBTileBytes;
            unsigned char* bt = sp + 2 * kATileBytes;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int c = lt + 128 * q;  // the chunks this thread loaded
                const int n = c >> 2, cc = c & 3;  // 16 weights k = 16cc .. 16cc+15 of row n
                const uint4 u = *reinterpret_cast<const uint4*>(rawb + n * 64 + cc * 16);
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int h = 0; h < 2; ++h) {  // two 16-byte chunks: k-chunk 2cc + h
                    uint4 o;
                    const float f[8] = {
                        (float)(int8_t)(w[2 * h] & 0xff),         (float)(int8_t)((w[2 * h] >> 8) & 0xff),
                        (float)(int8_t)((w[2 * h] >> 16) & 0xff), (float)(int8_t)(w[2 * h] >> 24),
                        (float)(int8_t)(w[2 * h + 1] & 0xff),     (float)(int8_t)((w[2 * h + 1] >> 8) & 0xff),
                        (float)(int8_t)((w[2 * h + 1] >> 16) & 0xff), (float)(int8_t)(w[2 * h + 1] >> 24)};
                    if (f16) {
                        o.x = pack_f16x2(f[0], f[1]); o.y = pack_f16x2(f[2], f[3]);
                        o.z = pack_f16x2(f[4], f[5]); o.w = pack_f16x2(f[6], f[7]);
                    } else {
                        o.x = pack_bf16x2(f[0], f[1]); o.y = pack_bf16x2(f[2], f[3]);
                        o.z = pack_bf16x2(f[4], f[5]); o.w = pack_bf16x2(f[6], f[7]);
                    }
                    const int kc = 2 * cc + h;
                    *reinterpret_cast<uint4*>(bt + n * 128 + ((kc ^ (n & 7)) << 4)) = o;
                }
            }
        };
        // Software pipeline: loads run kStagesTc - 1 tiles ahead of the conversions.
        for (int it = 0; it < KT + kStagesTc - 1 && ok; ++it) {
            if (it < KT) {
                const int st = it % kStagesTc;
                if (!mbar_wait(&empty[st], ((it / kStagesTc) & 1) ^ 1)) {
                    set_error(p.err, DEV_ERR_TIMEOUT);
                    ok = false;
                }
                if (ok) issue(it);
            }
            cp_async_commit();
            const int j = it - (kStagesTc - 1);
            if (j >= 0 && ok) {
                cp_async_wait<kStagesTc - 1>();
                convert(j);
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[j % kStagesTc]);
            }
        }
        cp_async_wait<0>();
        if (!ok) s_abort = 1;
        // ---- epilogue: this warp's 32 TMEM lanes = rows 32w .. 32w+31 of the tile ------------
        const bool got = mbar_wait(done, 0);
        if (!got) set_error(p.err, DEV_ERR_TIMEOUT);
        tc_fence_after();
        const int m = m0 + 32 * warp + lane;
#pragma unroll
        for (int c = 0; c < TBN; c += 32) {
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c, v);
            if (got && m < p.M) {
#pragma unroll
                for (int j = 0; j < 32; j += 2) epi_pair<EPI>(p, m, n0 + c + j, z, v[j], v[j + 1]);
            }
        }
    } else if (lane == 0) {
        // ---- MMA issuer ----------------------------------------------------------------------
        bool ok = true;
        int issued = 0;
        for (int kt = 0; kt < KT; ++kt) {
            const int st = kt % kStagesTc;
            if (!mbar_wait(&full[st], (kt / kStagesTc) & 1)) {
                set_error(p.err, DEV_ERR_TIMEOUT);
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sa = base + st * kStageTc;
            const uint64_t dhi = sw128_desc(sa), dlo = sw128_desc(sa + kATileBytes);
            const uint64_t db = sw128_desc(sa + 2 * kATileBytes);
            const uint32_t idesc = f16 ? kIdescF16 : kIdescBf16;
#pragma unroll
            for (int kk = 0; kk < TBK / 16; ++kk) {  // 32 bytes of K per MMA
                tc_mma(tmem, dhi + 2 * kk, db + 2 * kk, idesc, (kt | kk) ? 1u : 0u);
                if (has_lo) tc_mma(tmem, dlo + 2 * kk, db + 2 * kk, idesc, 1u);
            }
            tc_commit(&empty[st]);
            ++issued;
        }
        (void)ok;
        tc_commit(done);  // arrives once every MMA issued above has completed
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    }
}

template <int EPI>
void launch_tc_typed(const LinearArgs& a, cudaStream_t s) {
    static int configured = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured != dev) {
        cudaFuncSetAttribute(linear_tc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
        configured = dev;
    }
    dim3 grid(a.N / TBN, (a.M + TBM - 1) / TBM, a.splits);
    launch_k(linear_tc_kernel<EPI>, grid, dim3(kThreadsTc), kSmemTc, s, a);
}

}  // namespace

void launch_linear_tc(const LinearArgs& a, LinearEpi epi, cudaStream_t s) {
    switch (epi) {
        case EPI_F32: launch_tc_typed<EPI_F32>(a, s); break;
        case EPI_QKV: launch_tc_typed<EPI_QKV>(a, s); break;
        case EPI_RESID: launch_tc_typed<EPI_RESID>(a, s); break;
        case EPI_GELU: launch_tc_typed<EPI_GELU>(a, s); break;
        case EPI_PARTIAL: launch_tc_typed<EPI_PARTIAL>(a, s); break;
    }
}

}  // namespace ptts
