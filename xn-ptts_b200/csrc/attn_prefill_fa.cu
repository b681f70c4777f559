// Causal prefill attention on tcgen05, one CTA per (tile of up to 128 query rows of one sequence,
// group of kHeadsPerCta heads), sm_100a.
//
// Reference: the t > 1 branch of StreamingMultiheadAttention::forward (transformer.rs:231-248),
// softmax(q k^T * 1/sqrt(d) + mask) v with materialize_causal_mask (transformer.rs:94-108): the
// query at position p sees keys 0..=p of its stream.
//
// A CTA runs its heads' (head, 64-key tile) items as one pipeline, so the tensor cores always
// have the next item's work while the softmax of this one runs (a prompt of 32-512 rows has only
// 1-8 key tiles per head: one head per CTA left the chain S -> softmax -> P.V mostly idle).
//   warps 0-3   one query row per thread (TMEM lane 32 w + lane): write the head's q as bf16
//               hi/lo tiles (the next head's while this one runs), read S from TMEM, online
//               softmax in the exp2 domain with the causal mask, write P as bf16 hi/lo into TMEM
//               (tcgen05.st); O accumulates in TMEM, rescaled there only when a row's maximum
//               grows by more than 2^8; at each head's end O / l goes to the output row.
//   warp 4      lane 0 issues the MMAs (kind::f16, M = 128, N = 64, bf16):
//               S = Q_hi K^T + Q_lo K^T     A = Q (smem, K-major), B = K (smem, K-major)
//               O = P_hi V + P_lo V         A = P (TMEM), B = V (smem, MN-major)
//               S runs up to two items ahead of P.V (two S buffers in TMEM), across heads.
//   warp 5      lane 0 copies each item's K and V tiles (64 keys x one head, 128-byte swizzle)
//               with TMA into a two-slot ring.
// TMEM (256 columns): S0 0-63, S1 64-127, O 128-191, P hi 192-223, P lo 224-255
// (bf16 pairs, one row per lane). Keys past the tile's last position are masked in the softmax
// and their V rows zeroed before P.V (the slots may hold anything, and 0 x NaN is NaN). Every
// wait is bounded and sets DEV_ERR_TIMEOUT; a CTA that timed out waits, bounded, for its copies.
// Splitting q and P into hi + lo keeps the products f32-grade, as in the linears.
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int QT = 128;            // query rows per CTA
constexpr int KT = 64;             // keys per item
constexpr int kHeadsPerCta = 4;
constexpr int kThreadsF = 6 * 32;
constexpr int kQBytes = QT * 128;  // one plane of one head's q: 128 rows x 64 bf16
constexpr int kKVBytes = KT * 128; // one head's K (or V) tile
constexpr int kSlots = 2;          // K/V ring
// Shared layout (1024-aligned tiles): two Q buffers (hi, lo), the K/V ring (K, V per slot).
constexpr int kOffQ = 0;                               // buffer b: hi at b * 2 kQBytes, lo + kQBytes
constexpr int kOffKV = 2 * 2 * kQBytes;                // slot s: K at s * 2 kKVBytes, V + kKVBytes
constexpr int kOffBar = kOffKV + kSlots * 2 * kKVBytes;
constexpr int kSmemF = 1024 + kOffBar + 256;
static_assert(2 * (kSmemF + 1024) <= 228 * 1024, "two CTAs per SM");
constexpr uint32_t kTmemColsF = 256;
constexpr uint32_t kColO = 128, kColPh = 192, kColPl = 224;

// kind::f16, D f32, A/B bf16, M = 128, N = 64; kIdescPVf additionally marks B MN-major.
constexpr uint32_t kIdescSf = (1u << 4) | (1u << 7) | (1u << 10) | (8u << 17) | (8u << 24);
constexpr uint32_t kIdescPVf = kIdescSf | (1u << 16);

__device__ __forceinline__ uint64_t desc_k(uint32_t addr) {  // K-major SW128 (8-row groups 1024 B apart)
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr) {  // V: keys are rows, 64 dims per row
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)(8192 >> 4) << 16) |
           ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
__device__ __forceinline__ void fa_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fa_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fa_mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void fa_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void fa_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 consecutive TMEM columns of this warp's lanes, into registers / from registers.
__device__ __forceinline__ void fa_ld32(uint32_t taddr, float* v) {
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
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void fa_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void fa_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
        "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
        "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void fa_st8(uint32_t taddr, const uint32_t* r) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
__device__ __forceinline__ float fa_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ void fa_tma(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Write 64 f32 values of one row as bf16 hi/lo into two K-major SW128 tiles (row r).
__device__ __forceinline__ void q_row_hilo(unsigned char* hi, unsigned char* lo, int r, const float* v) {
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

// Barriers: K/V full and empty per slot, Q ready per buffer, S full and free per buffer, P full,
// O full.
struct FaBars {
    uint64_t kvfull[kSlots], kvempty[kSlots], qready[2], sfull[2], sfree[2], pfull, ofull;
};
static_assert(sizeof(FaBars) + 4 <= 256, "barriers fit the tail");

__global__ void __launch_bounds__(kThreadsF, 2) prefill_fa_kernel(PrefillArgs a, const int2* tiles,
                                                              const __grid_constant__ CUtensorMap tm_k,
                                                              const __grid_constant__ CUtensorMap tm_v,
                                                              int capacity) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* sm = smem_raw + (base - raw);
    FaBars* b = reinterpret_cast<FaBars*>(sm + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(b + 1);
    __shared__ int s_issued, s_consumed;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h0 = blockIdx.y * kHeadsPerCta;

    if (tid == 0) {
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(&b->kvfull[i], 1);
            mbar_init(&b->kvempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&b->qready[i], 4);
            mbar_init(&b->sfull[i], 1);
            mbar_init(&b->sfree[i], 4);
        }
        mbar_init(&b->pfull, 4);
        mbar_init(&b->ofull, 1);
        s_issued = 0;
        s_consumed = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemColsF)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    fa_before();
    __syncthreads();
    fa_after();
    const uint32_t tmem = *tmem_slot;
    grid_dep_wait();
    grid_dep_launch();

    const int2 tile = tiles[blockIdx.x];  // (first row, rows in tile)
    const int row0 = tile.x, nrows = tile.y;
    const int sid = a.row_stream[row0];
    const int pos_max = a.row_pos[row0 + nrows - 1];  // the tile's last row sees the most keys
    const bool bad = sid < 0 || pos_max < 0 || pos_max >= capacity;
    const int n_kt = bad ? 0 : (pos_max + KT) / KT;
    const int n_items = kHeadsPerCta * n_kt;  // item i: head h0 + i / n_kt, key tile i % n_kt

    if (warp < 4) {
        if (bad && tid == 0) set_error(a.err, DEV_ERR_BOUNDS);
        const int r = tid;  // this thread's query row in the tile (TMEM lane)
        const bool active = r < nrows;
        const int pos = active ? a.row_pos[row0 + r] : -1;
        const uint32_t lane_base = (uint32_t)(32 * warp) << 16;
        auto write_q = [&](int hh) {  // q of head h0 + hh into Q buffer hh % 2
            float q[64];
            const float* qr = a.q + ((long long)(row0 + (active ? r : 0)) * 8 + h0 + hh) * kHeadDim;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const float4 x = active ? *reinterpret_cast<const float4*>(qr + 4 * i) : make_float4(0.f, 0.f, 0.f, 0.f);
                q[4 * i] = x.x; q[4 * i + 1] = x.y; q[4 * i + 2] = x.z; q[4 * i + 3] = x.w;
            }
            unsigned char* qb = sm + kOffQ + (hh & 1) * 2 * kQBytes;
            q_row_hilo(qb, qb + kQBytes, r, q);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&b->qready[hh & 1]);
        };
        if (n_items > 0) write_q(0);
        // O accumulates in TMEM across a head's key tiles (P.V with accumulate). The exps of a
        // head are taken against m, raised lazily: only when a tile's row maximum exceeds m by
        // more than kRaise (log2 units) is O rescaled in TMEM and m raised, so P stays <= 2^kRaise
        // and the final O / l is the same softmax.
        constexpr float kRaise = 8.f;
        float m = -1e30f, l = 0.f;
        for (int i = 0; i < n_items; ++i) {
            const int hh = i / n_kt, kt = i - hh * n_kt;
            if (kt == 0) {
                m = -1e30f;
                l = 0.f;
                // The other Q buffer held head hh - 1, whose S products are all complete.
                if (hh + 1 < kHeadsPerCta) write_q(hh + 1);
            }
            // S(i) from TMEM: this thread's row, 64 keys; then the buffer goes back. A timeout
            // ends the warp's loop as a whole (the TMEM accesses below are warp-collective).
            if (!__all_sync(0xffffffffu, mbar_wait(&b->sfull[i & 1], (i >> 1) & 1))) {
                set_error(a.err, DEV_ERR_TIMEOUT);
                break;
            }
            fa_after();
            float s[64];
            fa_ld32(tmem + lane_base + (uint32_t)((i & 1) * 64), s);
            fa_ld32(tmem + lane_base + (uint32_t)((i & 1) * 64 + 32), s + 32);
            fa_wait_ld();
            fa_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&b->sfree[i & 1]);
            float mt = -INFINITY;
#pragma unroll
            for (int j = 0; j < 64; ++j) {
                const int key = kt * KT + j;
                s[j] = key <= pos ? s[j] * a.qscale : -INFINITY;
                mt = fmaxf(mt, s[j]);
            }
            // P.V of the previous item has read P and added into O (cheap by now: issued as soon
            // as that P was written).
            if (kt > 0 && !__all_sync(0xffffffffu, mbar_wait(&b->ofull, (i - 1) & 1))) {
                set_error(a.err, DEV_ERR_TIMEOUT);
                break;
            }
            fa_after();
            const bool raise = kt == 0 ? true : mt > m + kRaise;
            const float mnew = raise ? fmaxf(mt, m) : m;
            if (kt > 0 && __any_sync(0xffffffffu, raise)) {  // rescale O rows in TMEM (the whole warp)
                const float f = raise ? fa_exp2(m - mnew) : 1.f;
                l *= f;
                float ot[32];
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    fa_ld32(tmem + lane_base + kColO + 32 * half, ot);
                    fa_wait_ld();
                    uint32_t w[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(ot[j] * f);
                    fa_st32(tmem + lane_base + kColO + 32 * half, w);
                }
            }
            m = mnew;
            float rs = 0.f;
            // P(i) into TMEM, 16 keys (8 columns of bf16 pairs per plane) at a time.
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t ph[8], pl[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float e0 = fa_exp2(s[16 * c + 2 * j] - m), e1 = fa_exp2(s[16 * c + 2 * j + 1] - m);
                    rs += e0 + e1;
                    ph[j] = pack_bf16x2(e0, e1);
                    pl[j] = pack_bf16x2(e0 - bf16lo(ph[j]), e1 - bf16hi(ph[j]));
                }
                fa_st8(tmem + lane_base + kColPh + 8 * c, ph);
                fa_st8(tmem + lane_base + kColPl + 8 * c, pl);
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            l += rs;
            if (kt == n_kt - 1 && (kt + 1) * KT - 1 > pos_max) {
                // Zero the V rows past the tile's last key (read by P.V with P = 0).
                unsigned char* vt = sm + kOffKV + (i % kSlots) * 2 * kKVBytes + kKVBytes;
                const int first = pos_max + 1 - kt * KT;
                for (int c = first * 8 + tid; c < KT * 8; c += 128)
                    *reinterpret_cast<uint4*>(vt + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
                // Each warp's zeros precede its own arrival on pfull; P.V waits for all four.
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
            fa_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&b->pfull);
            if (kt < n_kt - 1) continue;
            // The head's last tile: O / l from TMEM into the output row (16-byte stores).
            if (!__all_sync(0xffffffffu, mbar_wait(&b->ofull, i & 1))) {
                set_error(a.err, DEV_ERR_TIMEOUT);
                break;
            }
            fa_after();
            const float inv = 1.f / l;
            const long long at = (long long)(row0 + r) * kRowWidth + (h0 + hh) * kHeadDim;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                float o[32];
                fa_ld32(tmem + lane_base + kColO + 32 * half, o);
                fa_wait_ld();
                if (!active) continue;
                const long long ah = at + 32 * half;
                if (a.out_mode == kOutF32) {
                    float4* out = reinterpret_cast<float4*>(static_cast<float*>(a.out) + ah);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        out[j] = make_float4(o[4 * j] * inv, o[4 * j + 1] * inv, o[4 * j + 2] * inv, o[4 * j + 3] * inv);
                } else if (a.out_mode == kOutBf16) {
                    uint4* out = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + ah);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        out[j] = make_uint4(pack_bf16x2(o[8 * j] * inv, o[8 * j + 1] * inv),
                                            pack_bf16x2(o[8 * j + 2] * inv, o[8 * j + 3] * inv),
                                            pack_bf16x2(o[8 * j + 4] * inv, o[8 * j + 5] * inv),
                                            pack_bf16x2(o[8 * j + 6] * inv, o[8 * j + 7] * inv));
                } else {
                    uint4* oh = reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + ah);
                    uint4* ol = reinterpret_cast<uint4*>(static_cast<__half*>(a.out_lo) + ah);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint4 h, lo4;
                        split_f16x2(o[8 * j] * inv, o[8 * j + 1] * inv, h.x, lo4.x);
                        split_f16x2(o[8 * j + 2] * inv, o[8 * j + 3] * inv, h.y, lo4.y);
                        split_f16x2(o[8 * j + 4] * inv, o[8 * j + 5] * inv, h.z, lo4.z);
                        split_f16x2(o[8 * j + 6] * inv, o[8 * j + 7] * inv, h.w, lo4.w);
                        oh[j] = h;
                        ol[j] = lo4;
                    }
                }
            }
        }
    } else if (warp == 4 && lane == 0) {
        // ---- MMA issuer ----------------------------------------------------------------------
        // Two independent streams of work, polled without blocking: S(i) once item i's K/V have
        // landed, its Q is written and its S buffer is free; P.V(i) once P(i) is in TMEM. S thus
        // runs up to two items ahead of P.V, across heads too. Bounded: no progress for
        // kWaitLimitCycles ends the loop with DEV_ERR_TIMEOUT.
        auto s_ready = [&](int i) {
            const int hh = i / n_kt;
            return mbar_test_wait(&b->kvfull[i % kSlots], (i / kSlots) & 1) &&
                   mbar_test_wait(&b->qready[hh & 1], (hh >> 1) & 1) &&
                   (i < 2 || mbar_test_wait(&b->sfree[i & 1], ((i >> 1) & 1) ^ 1));
        };
        auto issue_s = [&](int i) {
            const int hh = i / n_kt, slot = i % kSlots;
            fa_after();
            const uint32_t qa = base + kOffQ + (hh & 1) * 2 * kQBytes;
            const uint64_t dqh = desc_k(qa), dql = desc_k(qa + kQBytes);
            const uint64_t dk = desc_k(base + kOffKV + slot * 2 * kKVBytes);
            const uint32_t d = tmem + (uint32_t)((i & 1) * 64);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // head dim 64 = 4 x 16: 32 bytes per step
                fa_mma_ss(d, dqh + 2 * kk, dk + 2 * kk, kIdescSf, kk ? 1u : 0u);
                fa_mma_ss(d, dql + 2 * kk, dk + 2 * kk, kIdescSf, 1u);
            }
            fa_commit(&b->sfull[i & 1]);
        };
        auto issue_pv = [&](int i) {
            fa_after();
            const uint64_t dv = desc_mn(base + kOffKV + (i % kSlots) * 2 * kKVBytes + kKVBytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // 64 keys = 4 x 16: P 8 columns, V 2 x 1024 bytes
                // O accumulates over the head's key tiles; its first tile starts it afresh.
                fa_mma_ts(tmem + kColO, tmem + kColPh + 8 * kk, dv + 128 * kk, kIdescPVf,
                          (i % n_kt != 0 || kk) ? 1u : 0u);
                fa_mma_ts(tmem + kColO, tmem + kColPl + 8 * kk, dv + 128 * kk, kIdescPVf, 1u);
            }
            fa_commit(&b->ofull);
            fa_commit(&b->kvempty[i % kSlots]);  // S(i) and P.V(i) have read the slot
            s_consumed = i + 1;
        };
        int next_s = 0, next_pv = 0;
        long long t0 = clock64();
        while (next_pv < n_items) {
            bool progressed = false;
            if (next_s < n_items && s_ready(next_s)) {
                issue_s(next_s++);
                progressed = true;
            }
            if (next_pv < next_s && mbar_test_wait(&b->pfull, next_pv & 1)) {
                issue_pv(next_pv++);
                progressed = true;
            }
            if (progressed) {
                t0 = clock64();
            } else if (clock64() - t0 > kWaitLimitCycles) {
                set_error(a.err, DEV_ERR_TIMEOUT);
                break;
            } else {
                __nanosleep(20);  // leave the issue slots to the softmax warp sharing this SMSP
            }
        }
    } else if (warp == 5 && lane == 0) {
        // ---- K/V producer --------------------------------------------------------------------
        const long long row_base = (long long)sid * capacity;
        for (int i = 0; i < n_items; ++i) {
            const int hh = i / n_kt, kt = i - hh * n_kt, slot = i % kSlots;
            if (i >= kSlots && !mbar_wait(&b->kvempty[slot], ((i / kSlots) & 1) ^ 1)) {
                set_error(a.err, DEV_ERR_TIMEOUT);
                break;
            }
            const uint32_t dst = base + kOffKV + slot * 2 * kKVBytes;
            mbar_arrive_expect_tx(&b->kvfull[slot], 2 * kKVBytes);
            const int x = (h0 + hh) * kHeadDim, y = (int)(row_base + (long long)kt * KT);
            fa_tma(dst, &tm_k, x, y, &b->kvfull[slot]);
            fa_tma(dst + kKVBytes, &tm_v, x, y, &b->kvfull[slot]);
            s_issued = i + 1;
        }
    }
    fa_before();
    __syncthreads();
    if (tid == 0) {
        // Copies issued but never consumed (only after a timeout): let them land before exit.
        for (int i = s_consumed; i < s_issued; ++i) mbar_wait(&b->kvfull[i % kSlots], (i / kSlots) & 1);
    }
    if (warp == 0) {
        fa_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColsF) : "memory");
    }
}

}  // namespace

bool launch_prefill_attn_fa(const PrefillArgs& a, const int2* tiles, int n_tiles, int streams, int capacity,
                            cudaStream_t s) {
    const long long rows = (long long)streams * capacity;
    if (rows >= (1LL << 31)) return false;
    CUtensorMap mk, mv;
    if (!bf16_rows_map(&mk, a.k_cache, rows, kRowWidth, kHeadDim, KT) ||
        !bf16_rows_map(&mv, a.v_cache, rows, kRowWidth, kHeadDim, KT))
        return false;
    set_max_dynamic_smem(reinterpret_cast<const void*>(prefill_fa_kernel), kSmemF);
    launch_k(prefill_fa_kernel, dim3(n_tiles, (kRowWidth / kHeadDim) / kHeadsPerCta), dim3(kThreadsF), kSmemF, s, a,
             tiles, mk, mv, capacity);
    return true;
}

}  // namespace ptts
