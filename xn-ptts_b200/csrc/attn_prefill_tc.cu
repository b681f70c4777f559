// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
// Reference: the t > 1 branch of StreamingMultiheadAttention::forward (transformer.rs:231-248),
// softmax(q k^T * 1/sqrt(d) + mask) v with materialize_causal_mask (transformer.rs:94-108): the
// query at position p sees keys 0..=p of its stream.
//
// One CTA per (tile of up to 128 consecutive query rows of one sequence, head). 160 threads:
//   warps 0-3  one query row per thread (TMEM lane 32w + lane). They load the rotated q (f32)
//              as bf16 hi/lo tiles, cp.async each 64-key K and V tile of the head into
//              128-byte-swizzled shared memory, read S from TMEM, run the online softmax in the
//              exp2 domain with the causal mask, write P as bf16 hi/lo tiles, and fold each P.V
//              tile from TMEM into f32 register accumulators.
//   warp 4     one thread issues the MMAs (cta_group::1, kind::f16, M = 128, N = 64):
//              S = Q_hi K^T + Q_lo K^T   (A and B K-major, K = head dim)
//              O = P_hi V + P_lo V       (A K-major over keys, B = V MN-major)
// TMEM: S in columns 0..63, the P.V tile in 64..127. The four phases of a key tile hand over
// through mbarriers (kv -> S -> P -> O); every wait is bounded and sets DEV_ERR_TIMEOUT.
// Splitting q and P into hi + lo keeps products f32-grade, as in the linears.
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int QT = 128;            // query rows per CTA
constexpr int KT = 64;             // keys per tile
constexpr int kWarps = 5;
constexpr int kThreadsP = kWarps * 32;
constexpr int kQBytes = QT * 128;  // 64 bf16 per row
constexpr int kKVBytes = KT * 128;
constexpr int kPBytes = QT * 128;  // 64 keys per row
// Shared layout (1024-aligned tiles): Q_hi, Q_lo, two K/V buffers (K, V each), P_hi, P_lo,
// barriers, TMEM slot. Key tile kt uses buffer kt % 2, so the next tile's copies run while
// this one's MMAs and softmax do.
constexpr int kOffQh = 0, kOffQl = kQBytes, kOffK = 2 * kQBytes, kOffV = kOffK + kKVBytes;
constexpr int kKVBuf = 2 * kKVBytes;  // from one buffer's K to the next one's
constexpr int kOffPh = kOffK + 2 * kKVBuf, kOffPl = kOffPh + kPBytes;
constexpr int kOffBar = kOffPl + kPBytes;
constexpr int kSmemP = 1024 + kOffBar + 128;
constexpr uint32_t kTmemColsP = 128;

// kind::f16, D f32, A/B bf16, M = 128, N = 64; kIdescPV additionally marks B MN-major (bit 16).
constexpr uint32_t kIdescS = (1u << 4) | (1u << 7) | (1u << 10) | (8u << 17) | (8u << 24);
constexpr uint32_t kIdescPV = kIdescS | (1u << 16);

// K-major SW128 tile (rows of 128 B, 8-row groups 1024 B apart).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// MN-major SW128 tile of V: rows = keys (the K dimension), 64 dims (N) contiguous per row;
// groups of 8 keys 1024 B apart (stride byte offset), one 64-wide N group (leading byte offset
// unused).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(8192 >> 4) << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
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
__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Write 64 f32 values of one row as bf16 hi/lo into two K-major SW128 tiles (row r).
__device__ __forceinline__ void store_row_hilo(unsigned char* hi, unsigned char* lo, int r, const float* v) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 h, l;
        uint32_t* hp = &h.x;
        uint32_t* lp = &l.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float a = v[8 * c + 2 * e], b = v[8 * c + 2 * e + 1];
            hp[e] = pack_bf16x2(a, b);
            lp[e] = pack_bf16x2(a - bf16lo(hp[e]), b - bf16hi(hp[e]));
        }
        const int off = r * 128 + ((c ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(hi + off) = h;
        *reinterpret_cast<uint4*>(lo + off) = l;
    }
}

// Two CTAs per SM (shared memory allows two): ten warps put three on one SM sub-partition, whose
// 16K registers hold three warps only at 168 registers a thread or fewer (0 spills at 168).
__global__ void __maxnreg__(168) prefill_tc_kernel(PrefillArgs a, const int2* tiles) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* sm = smem_raw + (base - raw);
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + kOffBar);  // kv, s, p, o
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 4);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y;

    if (tid == 0) {
        mbar_init(&bar[0], 4);
        mbar_init(&bar[1], 1);
        mbar_init(&bar[2], 4);
        mbar_init(&bar[3], 1);
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemColsP)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t tmem = *tmem_slot;
    grid_dep_wait();
    grid_dep_launch();

    const int2 tile = tiles[blockIdx.x];  // (first row, rows in tile)
    const int row0 = tile.x, nrows = tile.y;
    const int sid = a.row_stream[row0];
    // The last row of a tile has the largest position: keys 0..=pos_max are read.
    const int pos_max = a.row_pos[row0 + nrows - 1];
    const long long cap_rows = a.stream_elems / kRowWidth;
    const bool bad = sid < 0 || pos_max < 0 || pos_max >= cap_rows;
    const int n_kt = bad ? 0 : (pos_max + KT) / KT;
    const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(a.k_cache) + (long long)sid * a.stream_elems + h * kHeadDim;
    const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(a.v_cache) + (long long)sid * a.stream_elems + h * kHeadDim;

    if (warp < 4) {
        if (bad && tid == 0) set_error(a.err, DEV_ERR_BOUNDS);
        const int r = tid;                    // this thread's query row in the tile
        const bool active = r < nrows;
        const int pos = active ? a.row_pos[row0 + r] : -1;
        bool ok = true;
        // K and V tiles of keys kt*64 .. kt*64+63 into buffer kt % 2: 64 rows x 8 chunks each,
        // 2 rows per thread, one cp.async group per tile.
        auto load_kv = [&](int kt) {
            const uint32_t buf = (uint32_t)((kt & 1) * kKVBuf);
#pragma unroll
            for (int i = 0; i < (KT * 8) / 128; ++i) {
                const int c = tid + 128 * i;
                const int kr = c >> 3, ch = c & 7;
                const int key = kt * KT + kr;
                const bool valid = key <= pos_max;
                const long long off = (long long)(valid ? key : 0) * kRowWidth + ch * 8;
                const uint32_t dst = buf + (uint32_t)(kr * 128 + ((ch ^ (kr & 7)) << 4));
                cp_async16(base + kOffK + dst, kc + off, valid);
                cp_async16(base + kOffV + dst, vc + off, valid);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
        };
        if (n_kt > 0) load_kv(0);
        // Q (rotated, f32) -> bf16 hi/lo tiles.
        {
            float q[64];
            const float* qr = a.q + (long long)(row0 + (active ? r : 0)) * a.ld + h * kHeadDim;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float4 x = active ? *reinterpret_cast<const float4*>(qr + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
                q[4 * i] = x.x; q[4 * i + 1] = x.y; q[4 * i + 2] = x.z; q[4 * i + 3] = x.w;
            }
            store_row_hilo(sm + kOffQh, sm + kOffQl, r, q);
        }
        float o[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) o[i] = 0.f;
        float m = -1e30f, l = 0.f;
        // Key tile kt: [S(kt) ready] softmax -> P(kt) -> [tile kt + 1's K/V landed: the MMA
        // thread computes S(kt + 1) right after P(kt).V] -> [P(kt).V ready] fold. The copies of
        // tile kt + 1 run during tile kt's softmax.
        float corr = 1.f;
        for (int kt = 0; kt < n_kt && ok; ++kt) {
            const uint32_t par = kt & 1;
            auto kv_ready = [&]() {  // this thread's copies so far have landed: tell the MMA thread
                asm volatile("cp.async.wait_group 0;" ::: "memory");
                fence_proxy_async();
                tc_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bar[0]);
            };
            if (kt == 0) kv_ready();  // tile 0 (and the Q tiles)
            // Tile kt + 1 goes to the other buffer, last read by tile kt - 1's MMAs, which are
            // complete: this thread waited for its P.V product at the end of the last iteration.
            if (kt + 1 < n_kt) load_kv(kt + 1);
            // S from TMEM: this thread's row, 64 keys.
            if (!mbar_wait(&bar[1], par)) {
                set_error(a.err, DEV_ERR_TIMEOUT);
                ok = false;
            }
            tc_after();
            float s[64];
            tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + 0u, s);
            tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + 32u, s + 32);
            float mt = m;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const int key = kt * KT + j;
                s[j] = key <= pos ? s[j] * a.qscale : -INFINITY;
                mt = fmaxf(mt, s[j]);
            }
            corr = fast_exp2(m - mt);
            float rs = 0.f;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                s[j] = fast_exp2(s[j] - mt);
                rs += s[j];
            }
            store_row_hilo(sm + kOffPh, sm + kOffPl, r, s);
            fence_proxy_async();
            tc_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bar[2]);
            if (kt + 1 < n_kt) kv_ready();
            // O tile from TMEM, folded into the running accumulator.
            if (ok && !mbar_wait(&bar[3], par)) {
                set_error(a.err, DEV_ERR_TIMEOUT);
                ok = false;
            }
            tc_after();
            float ot[64];
            tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + 64u, ot);
            tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + 96u, ot + 32);
#pragma unroll
            for (int i = 0; i < 64; ++i) o[i] = fmaf(o[i], corr, ot[i]);
            l = fmaf(l, corr, rs);
            m = mt;
            tc_before();
        }
        if (active && ok && n_kt > 0) {
            const float inv = 1.f / l;
            const long long at = (long long)(row0 + r) * a.ld + h * kHeadDim;
            if (a.out_mode == kOutF32) {
                float* out = static_cast<float*>(a.out) + at;
#pragma unroll
                for (int i = 0; i < 16; ++i)
                    *reinterpret_cast<float4*>(out + 4 * i) =
                        make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
            } else if (a.out_mode == kOutBf16) {
                uint32_t* oh = reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(a.out) + at);
#pragma unroll
                for (int i = 0; i < 32; ++i) oh[i] = pack_bf16x2(o[2 * i] * inv, o[2 * i + 1] * inv);
            } else {
                uint32_t* oh = reinterpret_cast<uint32_t*>(static_cast<__half*>(a.out) + at);
                uint32_t* ol = reinterpret_cast<uint32_t*>(static_cast<__half*>(a.out_lo) + at);
#pragma unroll
                for (int i = 0; i < 32; ++i) split_f16x2(o[2 * i] * inv, o[2 * i + 1] * inv, oh[i], ol[i]);
            }
        }
    } else if (lane == 0) {
        // MMA issuer.
        const uint64_t dqh = desc_kmajor(base + kOffQh), dql = desc_kmajor(base + kOffQl);
        const uint64_t dk0 = desc_kmajor(base + kOffK), dv0 = desc_mnmajor(base + kOffV);
        const uint64_t dk1 = desc_kmajor(base + kOffK + kKVBuf), dv1 = desc_mnmajor(base + kOffV + kKVBuf);
        const uint64_t dph = desc_kmajor(base + kOffPh), dpl = desc_kmajor(base + kOffPl);
        // S(kt) = Q K(kt)^T once tile kt's K/V have landed; P(kt).V once P(kt) is written, then
        // at once S(kt + 1), so that it runs while the warps fold P(kt).V.
        auto issue_s = [&](int kt) -> bool {
            if (!mbar_wait(&bar[0], kt & 1)) return false;
            tc_after();
            const uint64_t dk = (kt & 1) ? dk1 : dk0;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // head dim 64 = 4 x 16: 32 bytes per step
                tc_mma(tmem, dqh + 2 * kk, dk + 2 * kk, kIdescS, kk ? 1u : 0u);
                tc_mma(tmem, dql + 2 * kk, dk + 2 * kk, kIdescS, 1u);
            }
            tc_commit(&bar[1]);
            return true;
        };
        bool ok = n_kt == 0 || issue_s(0);
        for (int kt = 0; kt < n_kt && ok; ++kt) {
            const uint32_t par = kt & 1;
            if (!mbar_wait(&bar[2], par)) {
                ok = false;
                break;
            }
            tc_after();
            const uint64_t dv = (kt & 1) ? dv1 : dv0;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // 64 keys = 4 x 16: P 32 bytes, V 2 x 1024 bytes
                tc_mma(tmem + 64u, dph + 2 * kk, dv + 128 * kk, kIdescPV, kk ? 1u : 0u);
                tc_mma(tmem + 64u, dpl + 2 * kk, dv + 128 * kk, kIdescPV, 1u);
            }
            tc_commit(&bar[3]);
            if (kt + 1 < n_kt) ok = issue_s(kt + 1);
        }
        if (!ok) set_error(a.err, DEV_ERR_TIMEOUT);
    }
    tc_before();
    __syncthreads();
    if (warp == 0) {
        tc_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColsP) : "memory");
    }
}

}  // namespace

void launch_prefill_attn_tc(const PrefillArgs& a, const int2* tiles, int n_tiles, cudaStream_t s) {
    set_max_dynamic_smem(reinterpret_cast<const void*>(prefill_tc_kernel), kSmemP);
    launch_k(prefill_tc_kernel, dim3(n_tiles, kRowWidth / kHeadDim), dim3(kThreadsP), kSmemP, s, a, tiles);
}

}  // namespace ptts
