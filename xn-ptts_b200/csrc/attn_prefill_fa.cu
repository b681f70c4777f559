// Causal prefill attention on tcgen05, one CTA per (tile of up to 128 query rows of one sequence,
// group of 1, 2 or 4 heads: 8 / gridDim.y), sm_100a.
//
// Reference: the t > 1 branch of StreamingMultiheadAttention::forward (transformer.rs:231-248),
// softmax(q k^T * 1/sqrt(d) + mask) v with materialize_causal_mask (transformer.rs:94-108): the
// query at position p sees keys 0..=p of its stream.
//
// A CTA runs its heads' (head, 64-key tile) items as one pipeline, so the tensor cores always
// have the next item's work while the softmax of this one runs (a prompt of 32-512 rows has only
// 1-8 key tiles per head: one head per CTA left the chain S -> softmax -> P.V mostly idle).
//   warps 0-7   softmax: two threads per query row (row 32 (w % 4) + lane = TMEM lane, half
//               w / 4 of the keys and of the output dims). Read S from TMEM, online softmax in
//               the exp2 domain with the causal mask (the two halves of a row agree through one
//               barrier.red per item that the maximum stays, or exchange it through shared
//               memory when a head starts or it must be raised), write P as bf16 hi/lo into TMEM
//               (tcgen05.st) over the columns of S it came from; O accumulates in TMEM, rescaled
//               there only when a row's maximum grows by more than 2^8 (the one case in which
//               the softmax waits for the previous P.V); O / l of each head goes to the output
//               rows at the next item.
//   warp 8      lane 0 issues the MMAs (kind::f16, M = 128, N = 64, bf16):
//               S = Q_hi K^T + Q_lo K^T     A = Q (smem, K-major), B = K (smem, K-major)
//               O += P_hi V + P_lo V        A = P (TMEM), B = V (smem, MN-major)
//               Two S/P buffers in TMEM: S(i + 2) reuses buffer i % 2 once P.V(i) has read P(i)
//               from it, so S runs an item ahead of the softmax, across heads, and the softmax
//               of item i + 1 overlaps P.V(i). Two O buffers (head parity), so the softmax
//               writes out a head's O during the next head's first item instead of waiting at
//               the head's end for its last P.V.
//   warp 9      lane 0 copies with TMA each head's Q tiles (the bf16 hi/lo planes the q producer
//               wrote) and each item's K and V tiles (64 keys x one head, 128-byte swizzle) into
//               a two-slot K ring and a three-slot V ring: a K slot frees once its S product is
//               done, a V slot once its P.V is.
// TMEM (256 columns): S/P buffers 0-63 and 64-127, O buffers 128-191 and 192-255. In a buffer,
// S is f32 (column = key); P replaces it as bf16 pairs, each half of the keys within its own 32
// columns: hi of keys 32h + 0..31 in columns 32h + 0..15, lo in 32h + 16..31 (one row per lane),
// so a thread overwrites only the S values it has read itself. Keys past the tile's last position
// are masked in the softmax and their V rows zeroed before P.V (the slots may hold anything, and
// 0 x NaN is NaN). Every wait is bounded and sets DEV_ERR_TIMEOUT; a CTA that timed out waits,
// bounded, for its copies. Splitting q and P into hi + lo keeps the products f32-grade, as in the
// linears.
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int QT = 128;            // query rows per CTA
constexpr int KT = 64;             // keys per item
constexpr int kHeadsPerCtaMax = 4;  // heads per CTA for large grids; fewer when tiles are few
constexpr int kSoftWarps = 8;    // two per TMEM lane quarter (two threads per row)
constexpr int kMmaWarp = kSoftWarps, kLoadWarp = kSoftWarps + 1;
constexpr int kThreadsF = (kSoftWarps + 2) * 32;
constexpr int kQBytes = QT * 128;  // one plane of one head's q: 128 rows x 64 bf16
constexpr int kKVBytes = KT * 128; // one head's K (or V) tile
constexpr int kKSlots = 2;         // K ring
constexpr int kVSlots = 3;         // V ring (one per S/P buffer: item i's V is never two phases behind)
// Shared layout (1024-aligned tiles): two Q buffers (hi, lo), the K/V ring (K, V per slot).
constexpr int kOffQ = 0;                               // buffer b: hi at b * 2 kQBytes, lo + kQBytes
constexpr int kOffK = 2 * 2 * kQBytes;                 // K slot s at s * kKVBytes
constexpr int kOffV = kOffK + kKSlots * kKVBytes;      // V slot s at s * kKVBytes
constexpr int kOffBar = kOffV + kVSlots * kKVBytes;
constexpr int kSmemF = 1024 + kOffBar + 256;
constexpr int kStaticSmemF = 5 * 1024;  // s_xmax, s_xsum and the issue counters (4,112 bytes)
static_assert(2 * (kSmemF + kStaticSmemF + 1024) <= 228 * 1024, "two CTAs per SM");
constexpr uint32_t kTmemColsF = 256;
constexpr int kBufs = 2;  // S/P buffers in TMEM, 64 columns each
constexpr uint32_t kColO = 64 * kBufs;  // O of head hh at kColO + 64 (hh % 2)
static_assert(kColO + 2 * 64 <= kTmemColsF, "S/P buffers and two O buffers fit the allocation");

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
__device__ __forceinline__ float fa_max3(float x, float y, float z) {  // sm_100 three-input max
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(x), "f"(y), "f"(z));
    return r;
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

// Barriers: K and V full and empty per slot (separate rings: a K slot frees once its S product is
// done, a V slot once its P.V is), Q ready and free per buffer, S full and free per S/P buffer (free
// once the P.V that read its P is done), P full and P.V done per S/P buffer. Item i uses phase
// i / n of slot or buffer i % n of a ring of n. A parity wait takes an older phase of the same
// parity as done, so a waiter must know that the barrier is not two or more phases behind the one
// it asks for, nor past it. Here S(i) in TMEM means P.V(i - kBufs) is done (so V(i - kVSlots) has
// landed), and neither S(i + kBufs) nor V(i + kVSlots) can start before P.V(i), which needs the
// softmax warps' P(i): every wait below asks for a phase within one of the barrier's own.
struct FaBars {
    uint64_t kfull[kKSlots], kempty[kKSlots], vfull[kVSlots], vempty[kVSlots], qready[2], qfree[2], sfull[kBufs],
        sfree[kBufs], pfull[kBufs], ofull[kBufs];
};
static_assert(sizeof(FaBars) + 4 <= 256, "barriers fit the tail");

// Named barrier 1 + q over the two softmax warps of row quarter q (64 threads), returning
// whether `v` held in any of them: both leave a loop together.
template <int ID>
__device__ __forceinline__ bool pair_any_id(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.or.pred q, %2, 64, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(ID)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ bool pair_any(int quarter, bool v) {
    switch (quarter) {
        case 0: return pair_any_id<1>(v);
        case 1: return pair_any_id<2>(v);
        case 2: return pair_any_id<3>(v);
        default: return pair_any_id<4>(v);
    }
}

__global__ void __launch_bounds__(kThreadsF, 2) prefill_fa_kernel(PrefillArgs a, const int2* tiles,
                                                              const __grid_constant__ CUtensorMap tm_k,
                                                              const __grid_constant__ CUtensorMap tm_v,
                                                              const __grid_constant__ CUtensorMap tm_qh,
                                                              const __grid_constant__ CUtensorMap tm_ql,
                                                              int capacity) {
    extern __shared__ unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* sm = smem_raw + (base - raw);
    FaBars* b = reinterpret_cast<FaBars*>(sm + kOffBar);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(b + 1);
    __shared__ int s_k_issued, s_v_issued, s_q_issued;
    __shared__ float s_xmax[2][2][QT];  // [item parity][half][row]: the halves' row maxima
    __shared__ float s_xsum[2][2][QT];  // [head parity][half][row]: the halves' row sums
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int heads_per_cta = (kRowWidth / kHeadDim) / (int)gridDim.y;
    const int h0 = blockIdx.y * heads_per_cta;

    if (tid == 0) {
        for (int i = 0; i < kKSlots; ++i) {
            mbar_init(&b->kfull[i], 1);
            mbar_init(&b->kempty[i], 1);
        }
        for (int i = 0; i < kVSlots; ++i) {
            mbar_init(&b->vfull[i], 1);
            mbar_init(&b->vempty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&b->qready[i], 1);
            mbar_init(&b->qfree[i], 1);
        }
        for (int i = 0; i < kBufs; ++i) {
            mbar_init(&b->sfull[i], 1);
            mbar_init(&b->sfree[i], 1);
            mbar_init(&b->pfull[i], kSoftWarps);
            mbar_init(&b->ofull[i], 1);
        }
        s_k_issued = 0;
        s_v_issued = 0;
        s_q_issued = 0;
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
    const bool bad = sid < 0 || pos_max < 0 || pos_max >= capacity || a.q_hi == nullptr;
    const int n_kt = bad ? 0 : (pos_max + KT) / KT;
    const int n_items = heads_per_cta * n_kt;  // item i: head h0 + i / n_kt, key tile i % n_kt

    if (warp < kSoftWarps) {
        if (bad && tid == 0) set_error(a.err, DEV_ERR_BOUNDS);
        const int quarter = warp & 3, half = warp >> 2;
        const int r = 32 * quarter + lane;  // this thread's query row in the tile (TMEM lane)
        const bool active = r < nrows;
        const int pos = active ? a.row_pos[row0 + r] : -1;
        const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
        // O accumulates in TMEM across a head's key tiles (P.V with accumulate). The exps of a
        // head are taken against m, raised lazily: only when a tile's row maximum exceeds m by
        // more than kRaise (log2 units) is O rescaled in TMEM and m raised, so P stays <= 2^kRaise
        // and the final O / l is the same softmax. Both halves of a row keep the same m.
        constexpr float kRaise = 8.f;
        float m = -1e30f, l = 0.f;
        int pend_h = -1, pend_i = 0;  // a head whose O is still to be written, and its last item
        float pend_l = 0.f;
        for (int i = 0, hh = 0, kt = 0; i < n_items; ++i) {  // item i: head h0 + hh, key tile kt
            if (kt == 0) {
                m = -1e30f;
                l = 0.f;
            }
            // S(i) from TMEM: this thread's row, its 32 keys.
            const int buf = i % kBufs;
            const uint32_t ph_i = (uint32_t)(i / kBufs) & 1u;  // phase parity of item i's barriers
            bool ok = __all_sync(0xffffffffu, mbar_wait(&b->sfull[buf], ph_i));
            float s[32];
            float mt = -INFINITY;
            if (ok) {
                fa_after();
                fa_ld32(tmem + lane_base + (uint32_t)(buf * 64 + 32 * half), s);
                fa_wait_ld();
                // q came scaled by log2(e) / sqrt(D): S is in the exp2 domain already.
                const int key0 = kt * KT + 32 * half;
                if (!__all_sync(0xffffffffu, key0 + 31 <= pos)) {  // some key of this half is masked
#pragma unroll
                    for (int j = 0; j < 32; ++j) s[j] = key0 + j <= pos ? s[j] : -INFINITY;
                }
                float m4[4];  // four independent chains of three-input maxima over 8 keys each
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float* sq = s + 8 * q;
                    m4[q] = fa_max3(fa_max3(fa_max3(sq[0], sq[1], sq[2]), sq[3], sq[4]), sq[5], sq[6]);
                    m4[q] = fmaxf(m4[q], sq[7]);
                }
                mt = fmaxf(fa_max3(m4[0], m4[1], m4[2]), m4[3]);
            }
            // One barrier.red over the row quarter's two warps: unless a head starts, a wait
            // timed out, or some row's maximum passed m + kRaise, m stays and nothing is
            // exchanged. Otherwise the halves exchange their maxima (and timeouts) and raise m.
            if (pair_any(quarter, !ok || kt == 0 || mt > m + kRaise)) {
                s_xmax[i & 1][half][r] = mt;
                if (pair_any(quarter, !ok)) {
                    set_error(a.err, DEV_ERR_TIMEOUT);
                    break;
                }
                mt = fmaxf(mt, s_xmax[i & 1][half ^ 1][r]);
                fa_after();
                const bool raise = kt == 0 ? true : mt > m + kRaise;
                const float mnew = raise ? fmaxf(mt, m) : m;
                if (kt > 0 && __any_sync(0xffffffffu, raise)) {  // rescale this half of O in TMEM
                    // O must hold P.V(i - 1) first (its commit follows every earlier P.V). The
                    // partner warp (same rows, same maxima) takes this branch too, so both agree
                    // on a timeout.
                    const bool done =
                        __all_sync(0xffffffffu, mbar_wait(&b->ofull[(i - 1) % kBufs], ((i - 1) / kBufs) & 1));
                    if (pair_any(quarter, !done)) {
                        set_error(a.err, DEV_ERR_TIMEOUT);
                        break;
                    }
                    fa_after();
                    const float f = raise ? fa_exp2(m - mnew) : 1.f;
                    l *= f;
                    float ot[32];
                    const uint32_t ocol = kColO + 64 * (hh & 1) + 32 * half;
                    fa_ld32(tmem + lane_base + ocol, ot);
                    fa_wait_ld();
                    uint32_t w[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(ot[j] * f);
                    fa_st32(tmem + lane_base + ocol, w);
                }
                m = mnew;
            }
            // P(i) into TMEM over this half's S columns: its 32 keys, 16 columns of bf16 pairs per
            // plane (hi, then lo). Only this thread's own lane and columns, already read. Pairs
            // of keys go through the packed f32x2 add and fma: s - m, the row sum (two chains)
            // and lo = e - hi (exact: one rounding of an exact difference).
            const uint32_t pcol = (uint32_t)(buf * 64 + 32 * half);
            const float2 neg_m = make_float2(-m, -m), minus1 = make_float2(-1.f, -1.f);
            float2 sum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                uint32_t ph[8], pl[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float2 x = __fadd2_rn(make_float2(s[16 * c + 2 * j], s[16 * c + 2 * j + 1]), neg_m);
                    const float2 e = make_float2(fa_exp2(x.x), fa_exp2(x.y));
                    sum[j & 1] = __fadd2_rn(sum[j & 1], e);
                    ph[j] = pack_bf16x2(e.x, e.y);
                    const float2 lo = __ffma2_rn(make_float2(bf16lo(ph[j]), bf16hi(ph[j])), minus1, e);
                    pl[j] = pack_bf16x2(lo.x, lo.y);
                }
                fa_st8(tmem + lane_base + pcol + 8 * c, ph);
                fa_st8(tmem + lane_base + pcol + 16 + 8 * c, pl);
            }
            l += (sum[0].x + sum[1].x) + (sum[0].y + sum[1].y);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            if (kt == n_kt - 1 && (kt + 1) * KT - 1 > pos_max) {
                // Zero the V rows past the tile's last key (read by P.V with P = 0), once V(i)
                // has landed (its copy runs apart from K's).
                if (!mbar_wait(&b->vfull[i % kVSlots], (i / kVSlots) & 1)) set_error(a.err, DEV_ERR_TIMEOUT);
                unsigned char* vt = sm + kOffV + (i % kVSlots) * kKVBytes;
                const int first = pos_max + 1 - kt * KT;
                for (int c = first * 8 + tid; c < KT * 8; c += 32 * kSoftWarps)
                    *reinterpret_cast<uint4*>(vt + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
                // Each warp's zeros precede its own arrival on pfull; P.V waits for all of them.
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
            fa_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&b->pfull[buf]);
            // Heads to write out now: the one pending from the previous item (its last P.V has
            // had the time of a softmax pass), then this one if it ends the CTA's work; a head
            // that ends earlier waits for the next item. O of head hh lives in O buffer hh % 2,
            // which the first P.V of head hh + 2 overwrites: that needs this warp's P of it, so
            // comes after the write-out.
            bool stop = false;
            for (int pass = 0; pass < 2; ++pass) {
                int fh, fi;
                float fl;
                if (pass == 0) {
                    if (pend_h < 0) continue;
                    fh = pend_h, fi = pend_i, fl = pend_l;
                    pend_h = -1;
                } else {
                    if (kt != n_kt - 1) break;
                    if (i < n_items - 1) {
                        pend_h = hh, pend_i = i, pend_l = l;
                        break;
                    }
                    fh = hh, fi = i, fl = l;
                }
                // The row sum over both halves, then O / l into this half of the output row
                // (16-byte stores). P.V(fi) done: S(i) in TMEM means P.V(i - kBufs) is done, so
                // the barrier is within one phase of it.
                ok = __all_sync(0xffffffffu, mbar_wait(&b->ofull[fi % kBufs], (fi / kBufs) & 1));
                s_xsum[fh & 1][half][r] = fl;  // slot fh % 2: heads fh and fh + 1 may share an item
                if (pair_any(quarter, !ok)) {
                    set_error(a.err, DEV_ERR_TIMEOUT);
                    stop = true;
                    break;
                }
                const float inv = 1.f / (fl + s_xsum[fh & 1][half ^ 1][r]);
                fa_after();
                float o[32];
                fa_ld32(tmem + lane_base + kColO + 64 * (fh & 1) + 32 * half, o);
                fa_wait_ld();
                if (!active) continue;
                const long long at = (long long)(row0 + r) * a.ld + (h0 + fh) * kHeadDim + 32 * half;
                if (a.out_mode == kOutF32) {
                    float4* out = reinterpret_cast<float4*>(static_cast<float*>(a.out) + at);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        out[j] = make_float4(o[4 * j] * inv, o[4 * j + 1] * inv, o[4 * j + 2] * inv,
                                             o[4 * j + 3] * inv);
                } else if (a.out_mode == kOutBf16) {
                    uint4* out = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(a.out) + at);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        out[j] = make_uint4(pack_bf16x2(o[8 * j] * inv, o[8 * j + 1] * inv),
                                            pack_bf16x2(o[8 * j + 2] * inv, o[8 * j + 3] * inv),
                                            pack_bf16x2(o[8 * j + 4] * inv, o[8 * j + 5] * inv),
                                            pack_bf16x2(o[8 * j + 6] * inv, o[8 * j + 7] * inv));
                } else {
                    uint4* oh = reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + at);
                    uint4* ol = reinterpret_cast<uint4*>(static_cast<__half*>(a.out_lo) + at);
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
            if (stop) break;
            if (++kt == n_kt) kt = 0, ++hh;
        }
    } else if (warp == kMmaWarp && lane == 0) {
        // ---- MMA issuer ----------------------------------------------------------------------
        // A fixed order, S(0 .. kBufs - 1), then per item i: P.V(i) once P(i) is in TMEM and V(i)
        // has landed, S(i + kBufs) once its K has landed, its Q is in and P.V(i) has freed the
        // buffer. Every wait suspends the thread instead of polling: this warp shares its SM
        // sub-partition with two softmax warps of each CTA, whose issue slots a polling loop
        // would take. Bounded: a wait that gives up ends the loop with DEV_ERR_TIMEOUT.
        auto wait_s = [&](int i) {
            const int hh = i / n_kt;
            return mbar_wait(&b->kfull[i % kKSlots], (i / kKSlots) & 1) &&
                   mbar_wait(&b->qready[hh & 1], (hh >> 1) & 1) &&
                   (i < kBufs || mbar_wait(&b->sfree[i % kBufs], ((i / kBufs) & 1) ^ 1));
        };
        auto issue_s = [&](int i) {
            const int hh = i / n_kt, slot = i % kKSlots;
            fa_after();
            const uint32_t qa = base + kOffQ + (hh & 1) * 2 * kQBytes;
            const uint64_t dqh = desc_k(qa), dql = desc_k(qa + kQBytes);
            const uint64_t dk = desc_k(base + kOffK + slot * kKVBytes);
            const uint32_t d = tmem + (uint32_t)((i % kBufs) * 64);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // head dim 64 = 4 x 16: 32 bytes per step
                fa_mma_ss(d, dqh + 2 * kk, dk + 2 * kk, kIdescSf, kk ? 1u : 0u);
                fa_mma_ss(d, dql + 2 * kk, dk + 2 * kk, kIdescSf, 1u);
            }
            fa_commit(&b->sfull[i % kBufs]);
            fa_commit(&b->kempty[slot]);  // S(i) has read the K slot
            if (i % n_kt == n_kt - 1) fa_commit(&b->qfree[hh & 1]);  // the head's Q tiles are read
        };
        auto issue_pv = [&](int i) {
            fa_after();
            const uint64_t dv = desc_mn(base + kOffV + (i % kVSlots) * kKVBytes);
            const uint32_t pb = tmem + (uint32_t)((i % kBufs) * 64);
            const uint32_t od = tmem + kColO + 64 * (uint32_t)((i / n_kt) & 1);  // the head's O
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // 64 keys = 4 x 16: P 8 columns, V 2 x 1024 bytes
                // Keys 16 kk.. of P: half kk / 2 of the buffer, its hi columns 8 (kk % 2) on, lo 16 on.
                const uint32_t ph = pb + 32 * (kk >> 1) + 8 * (kk & 1);
                // O accumulates over the head's key tiles; its first tile starts it afresh.
                fa_mma_ts(od, ph, dv + 128 * kk, kIdescPVf, (i % n_kt != 0 || kk) ? 1u : 0u);
                fa_mma_ts(od, ph + 16, dv + 128 * kk, kIdescPVf, 1u);
            }
            fa_commit(&b->ofull[i % kBufs]);
            fa_commit(&b->vempty[i % kVSlots]);  // P.V(i) has read the V slot
            fa_commit(&b->sfree[i % kBufs]);     // ... and P(i): the buffer takes S(i + kBufs)
        };
        bool ok = true;
        for (int i = 0; i < kBufs && i < n_items && ok; ++i)
            if ((ok = wait_s(i))) issue_s(i);
        for (int i = 0; i < n_items && ok; ++i) {
            ok = mbar_wait(&b->pfull[i % kBufs], (i / kBufs) & 1) &&
                 mbar_wait(&b->vfull[i % kVSlots], (i / kVSlots) & 1);
            if (!ok) break;
            issue_pv(i);
            if (i + kBufs < n_items && (ok = wait_s(i + kBufs))) issue_s(i + kBufs);
        }
        if (!ok) set_error(a.err, DEV_ERR_TIMEOUT);
    } else if (warp == kLoadWarp && lane == 0) {
        // ---- Q, K and V producer ------------------------------------------------------------
        const long long row_base = (long long)sid * capacity;
        // Q tiles of head hh (hi, lo: 128 rows x 64 bf16 from row0) into buffer hh % 2, once the
        // S products of head hh - 2 that read it are done.
        auto load_q = [&](int hh) -> bool {
            const int qb = hh & 1;
            if (hh >= 2 && !mbar_wait(&b->qfree[qb], ((hh >> 1) & 1) ^ 1)) return false;
            const uint32_t dst = base + kOffQ + qb * 2 * kQBytes;
            mbar_arrive_expect_tx(&b->qready[qb], 2 * kQBytes);
            fa_tma(dst, &tm_qh, (h0 + hh) * kHeadDim, row0, &b->qready[qb]);
            fa_tma(dst + kQBytes, &tm_ql, (h0 + hh) * kHeadDim, row0, &b->qready[qb]);
            s_q_issued = hh + 1;
            return true;
        };
        // K(j) then V(j - 1): K runs an item ahead of V, its slots freed by S alone.
        auto load_k = [&](int i) -> bool {
            const int hh = i / n_kt, kt = i - hh * n_kt, slot = i % kKSlots;
            if (i >= kKSlots && !mbar_wait(&b->kempty[slot], ((i / kKSlots) & 1) ^ 1)) return false;
            mbar_arrive_expect_tx(&b->kfull[slot], kKVBytes);
            fa_tma(base + kOffK + slot * kKVBytes, &tm_k, (h0 + hh) * kHeadDim,
                   (int)(row_base + (long long)kt * KT), &b->kfull[slot]);
            s_k_issued = i + 1;
            return true;
        };
        auto load_v = [&](int i) -> bool {
            const int hh = i / n_kt, kt = i - hh * n_kt, slot = i % kVSlots;
            if (i >= kVSlots && !mbar_wait(&b->vempty[slot], ((i / kVSlots) & 1) ^ 1)) return false;
            mbar_arrive_expect_tx(&b->vfull[slot], kKVBytes);
            fa_tma(base + kOffV + slot * kKVBytes, &tm_v, (h0 + hh) * kHeadDim,
                   (int)(row_base + (long long)kt * KT), &b->vfull[slot]);
            s_v_issued = i + 1;
            return true;
        };
        int q_loaded = 0;  // heads whose Q tiles are requested
        bool ok = n_items == 0 || load_q(0);
        q_loaded = 1;
        for (int i = 0; i <= n_items && ok; ++i) {
            if (i < n_items) {
                const int hh = i / n_kt, kt = i - hh * n_kt;
                if (kt == 0 && hh + 1 < heads_per_cta && q_loaded == hh + 1) {
                    ok = load_q(hh + 1);
                    q_loaded = hh + 2;
                }
                ok = ok && load_k(i);
            }
            if (ok && i >= 1) ok = load_v(i - 1);
        }
        if (!ok) set_error(a.err, DEV_ERR_TIMEOUT);
    }
    fa_before();
    __syncthreads();
    if (tid == 0) {
        // The last copies issued into each slot (consumed or not; a completed phase returns at
        // once): let them land before exit.
        for (int i = s_k_issued > kKSlots ? s_k_issued - kKSlots : 0; i < s_k_issued; ++i)
            mbar_wait(&b->kfull[i % kKSlots], (i / kKSlots) & 1);
        for (int i = s_v_issued > kVSlots ? s_v_issued - kVSlots : 0; i < s_v_issued; ++i)
            mbar_wait(&b->vfull[i % kVSlots], (i / kVSlots) & 1);
        // The Q copies: the last request of each buffer (a completed phase returns at once).
        for (int hh = s_q_issued > 2 ? s_q_issued - 2 : 0; hh < s_q_issued; ++hh)
            mbar_wait(&b->qready[hh & 1], (hh >> 1) & 1);
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
    CUtensorMap mk, mv, mqh, mql;
    if (!bf16_rows_map(&mk, a.k_cache, rows, kRowWidth, kHeadDim, KT) ||
        !bf16_rows_map(&mv, a.v_cache, rows, kRowWidth, kHeadDim, KT))
        return false;
    if (a.q_hi) {
        if (!bf16_rows_map(&mqh, a.q_hi, a.rows, kRowWidth, kHeadDim, QT, a.ld) ||
            !bf16_rows_map(&mql, a.q_lo, a.rows, kRowWidth, kHeadDim, QT, a.ld))
            return false;
    } else {
        mqh = mk;  // unused: the softmax warps convert the f32 q
        mql = mk;
    }
    set_max_dynamic_smem(reinterpret_cast<const void*>(prefill_fa_kernel), kSmemF);
    // Four heads per CTA give each CTA a long pipeline; with few tiles (short prompts), fewer
    // heads per CTA keep the SMs busy: two CTAs per SM want at least 2 x SMs CTAs.
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int hpc = kHeadsPerCtaMax;
    while (hpc > 1 && (long long)n_tiles * ((kRowWidth / kHeadDim) / hpc) < 2LL * sms) hpc /= 2;
    launch_k(prefill_fa_kernel, dim3(n_tiles, (kRowWidth / kHeadDim) / hpc), dim3(kThreadsF), kSmemF, s, a,
             tiles, mk, mv, mqh, mql, capacity);
    return true;
}

}  // namespace ptts
