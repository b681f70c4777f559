// int8-weight linears on the 5th-generation tensor cores (tcgen05 + TMEM), fed by TMA, sm_100a.
//
// Same contract as linear.cu (LinearArgs, the epilogues, split-K slices). Three weight forms:
//   kW8    the layer's int8 weights themselves (the default for int8 layers), copied by TMA as
//          int8 and widened in registers to the 16-bit type of the activations (f16 for the
//          layer stack's hi/lo planes, bf16 for a single bf16 plane) in the 128-byte-swizzled
//          K-major layout the MMA reads; int8 values are exact in both types, and the per-row
//          scale is applied to the f32 accumulator in the epilogue;
//   kW16   one 16-bit plane read as it is (the flow net's bf16 weights, a prompt's weights
//          widened once per call, or an f16 copy made at load time with PTTS_B200_WEIGHTS=f16);
//   kW16Lo two 16-bit planes (hi, lo) for f32 and q8_0 layers and the flow net's f32 weights.
//
// Roles are swapped against the row-major view: the MMA's M side (128 TMEM lanes) is 128 output
// features and its N side is RT activation rows, D^T[f][r] = sum_k W[f][k] X[r][k]. Per 16 k
// that is one tcgen05.mma.cta_group::1.kind::f16 per activation plane (hi, lo) with A = the
// weight tile and B = the activation tile, both K-major. Kernels:
//   linear_tma_kernel    one 128-feature x 32-row tile per CTA (decode sizes up to 4095 rows:
//                        a 512-row batch gives (N / 128) x 16 CTAs);
//   linear_persist_kernel prompts of 4096+ rows: one CTA per SM over all 128 x 128 tiles.
//
// linear_tma_kernel CTA: 512 threads (16 warps).
//   thread 0:   TMA producer over a kStages ring of {W 128x64, X hi RTx64, X lo RTx64} tiles,
//               weights and activations on separate barriers. The weight tiles of the first
//               stages are requested before the wait on the grid that wrote X (weights never
//               change), so with kW8 they are also widened before that wait ends.
//   thread 32:  MMA issuer; tcgen05.commit frees each stage and finally signals `done`.
//   warps 4-11: kW8 only: the converters (widen_w8: the 8 KB int8 tile lands in the upper half of
//               the stage's 16 KB weight slot and is widened in place).
//   all warps:  epilogue (drain_tile): warp w reads TMEM lanes 32 (w % 4) .. + 31 (features
//               n0 + 32 (w % 4) + lane), 8 rows per tcgen05.ld, into a shared-memory tile; then
//               each warp takes 2 whole rows, lane l the features 4l..4l+3, so stores are 16
//               bytes and RoPE pairs in-lane. Sixteen warps instead of four cut each warp's
//               serial share of the epilogue (GELU, RoPE), which bounds the decode-size launches.
// Every wait is bounded (DEV_ERR_TIMEOUT); after a timeout the CTA still waits, bounded, for the
// copies it issued and frees its TMEM. No clusters, no multicast.
#include <cuda.h>

#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int FT = 128;  // output features per CTA (MMA M)
constexpr int KS = 64;   // k per stage: one 128-byte swizzle row of f16
// 16 warps: the MMA-side roles take threads 0 and 32; all sixteen run the epilogue, four per
// TMEM lane quarter (warp w reads lanes 32 (w % 4) ..), each then storing 2 of the 32 staged rows.
constexpr int kEpiWarps = 16;
constexpr int kThreadsTma = 32 * kEpiWarps;
constexpr int kRowsPerWarp = 32 / kEpiWarps;

// Weight forms (see the top of this file).
enum : int { kW16 = 0, kW16Lo = 1, kW8 = 2 };
constexpr int kConvWarps = 8;   // kW8 converter warps
constexpr int kConvBar = 2;     // their named barrier (0: __syncthreads, 1: persistent epilogue)

template <int RT, int WM>
struct TmaTile {
    // 3 stages: a decode tile (RT 32, 74 KB) fits beside the decode attention's compact ring
    // (137 KB) on one SM, and two prompt tiles (RT 64, 97 KB) share an SM, so that one's epilogue
    // overlaps the other's loads and MMAs. A decode tile with a weight lo plane (40 KB a stage)
    // takes 2 stages (81 KB) for the same reason: with 3 (121 KB) a two-lane step's linears
    // waited for the other lane's attention to leave the SMs.
    static constexpr int kStages = (WM == kW16Lo && RT <= 32) ? 2 : ((WM == kW16Lo || RT <= 64) ? 3 : 4);
    static constexpr int kWBytes = FT * KS * 2;  // 16 KB per 16-bit weight plane
    static constexpr int kXBytes = RT * KS * 2;  // per activation plane
    static constexpr int kStageBytes = (WM == kW16Lo ? 2 : 1) * kWBytes + 2 * kXBytes;
    static constexpr int kXOffset = (WM == kW16Lo ? 2 : 1) * kWBytes;  // X hi, then X lo
    static constexpr int kBarOffset = kStages * kStageBytes;
    static constexpr int kSmem = 1024 + kBarOffset + 256;  // + alignment slack + barriers
    // Weight bytes a stage's copies deliver: the int8 tile (kW8) or the 16-bit plane(s).
    static constexpr uint32_t kWTx = WM == kW8 ? FT * KS : (WM == kW16Lo ? 2 : 1) * kWBytes;
    // Accumulator columns: RT rows of the hi plane, then RT rows of the lo plane (one N = 2 RT
    // MMA covers both, see linear_tma_kernel).
    static constexpr uint32_t kTmemCols = 2 * RT;
    static_assert(RT % 32 == 0 && RT >= 32 && RT <= 128, "RT: 32..128 in steps of 32");
    static_assert(kStageBytes % 1024 == 0, "stages stay 1024-byte aligned");
    static_assert(32 * (FT + 4) * 4 <= kBarOffset, "the QKV staging tile fits in the ring");
    static_assert(4 * kStages * 8 + 8 + 4 <= 256, "barriers fit the tail");
};

// Named barrier `ID` over N threads that returns whether `v` held in any of them (one answer for
// all, so a group leaves a loop together).
template <int ID, int N>
__device__ __forceinline__ bool bar_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(ID), "n"(N)
        : "memory");
    return r != 0;
}

// kW8: widen the int8 tile at the upper half of the 16 KB weight slot `w16` (128 rows x 64
// bytes, dense, as the TMA copied it) in place into the 128-byte-swizzled K-major 16-bit tile
// (128 rows x 128 bytes: the 16-byte chunk c of row r at chunk c ^ (r % 8)) that the MMA reads.
// Converter thread t (0..255) takes the 16-byte int8 chunks q = t + 256 i, i < 2 (row q / 4,
// k 16 (q % 4) .. + 15): the loads are contiguous, and each quarter-warp's stores hit the eight
// distinct 16-byte bank groups. The int8 tile is the slot's upper half, so every converter loads
// its share before any stores: one named barrier between them, which is also where the
// converters agree on the wait for the tile (`landed`: false in any of them, and all return
// false together, so none is left at a barrier). The proxy fence then makes the stores visible
// to the tensor core.
template <bool F16>
__device__ __forceinline__ bool widen_w8(unsigned char* w16, int t, bool landed) {
    constexpr int kChunks = FT * KS / 16 / (32 * kConvWarps);  // 16-byte int8 chunks per thread
    const unsigned char* w8 = w16 + FT * KS;
    uint4 in[kChunks];
#pragma unroll
    for (int i = 0; i < kChunks; ++i) in[i] = *reinterpret_cast<const uint4*>(w8 + 16 * (t + 32 * kConvWarps * i));
    if (bar_any<kConvBar, 32 * kConvWarps>(!landed)) return false;
#pragma unroll
    for (int i = 0; i < kChunks; ++i) {
        const int q = t + 32 * kConvWarps * i, r = q >> 2, j = q & 3;
        uint4 a, b;
        i8x4_convert<F16>(in[i].x, a.x, a.y);
        i8x4_convert<F16>(in[i].y, a.z, a.w);
        i8x4_convert<F16>(in[i].z, b.x, b.y);
        i8x4_convert<F16>(in[i].w, b.z, b.w);
        unsigned char* row = w16 + r * 128;
        *reinterpret_cast<uint4*>(row + (((2 * j) ^ (r & 7)) << 4)) = a;
        *reinterpret_cast<uint4*>(row + (((2 * j + 1) ^ (r & 7)) << 4)) = b;
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    return true;
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B both f16 (formats 0) or both
// bf16 (format 1 at bits 7-9 and 10-12), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
template <int RT>
constexpr uint32_t idesc_f16() {
    return (1u << 4) | ((uint32_t)(RT >> 3) << 17) | ((uint32_t)(FT >> 4) << 24);
}
template <int RT>
constexpr uint32_t idesc_bf16() {
    return idesc_f16<RT>() | (1u << 7) | (1u << 10);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile at `addr` (1024-aligned):
// start >> 4 in bits 0-13, leading byte offset 1 (unused when swizzled), stride byte offset
// 1024 B (8 rows of 128 B) >> 4 in bits 32-45, version 1 at bit 46, SWIZZLE_128B (2) at 61-63.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D (TMEM) += A (smem) x B (smem), or D = A x B when accumulate is 0.
__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives on `bar` once every MMA this thread issued before has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 consecutive f32 columns of this thread's TMEM lane.
// 8 consecutive TMEM columns of this warp's 32 lanes (tcgen05.ld.32x32b.x8).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, float (&v)[N]) {
    static_assert(N == 8, "the epilogues read 8 columns at a time");
    tmem_ld8(taddr, v);
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 2-D tiled TMA load of the box at (x = k, y = row) into shared memory, completing its bytes on
// `bar`. x is a multiple of 64 f16 (128 bytes), so the 16-byte rule on x always holds.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                 uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ float gelu_tc(float x, int tanh_form) {
    if (tanh_form) {
        const float u2 = (x * x * 0.07135482f + 1.595769f) * x;
        return x / (1.0f + expf(-u2));
    }
    return gelu_erf(x);
}

// Staged tile row stride in floats: 128 features + 4 (keeps float4 alignment, spreads banks).
constexpr int kStageStride = FT + 4;

// EPI_QKV of 32 staged rows: st[j * kStageStride + c] = accumulator of row mbase + j, tile
// feature c. Warp w takes rows w, w + 8, ..., lane l features n0 + 4l .. 4l + 3, i.e. the RoPE
// pairs (4l, 4l+1) and (4l+2, 4l+3) (rope.rs:37-95), with the arithmetic of linear.cu's qkv_pair.
// Row metadata and every RoPE entry are loaded before the first store.
__device__ __forceinline__ void qkv_rows(const LinearArgs& p, const float* st, int n0, int mbase,
                                         int warp = threadIdx.x >> 5) {
    const int lane = threadIdx.x & 31;
    const int hd = p.heads * kHeadDim, kvd = p.kv_heads * kHeadDim;
    const int f = n0 + 4 * lane, d = f % kHeadDim;
    const int region = f < hd ? 0 : (f < hd + kvd ? 1 : 2);
    const int group = p.heads / p.kv_heads;
    const float4 sc = __ldg(reinterpret_cast<const float4*>(p.scale + f));
    const int ml = mbase + lane;
    const int pos_l = ml < p.M ? __ldg(p.row_pos + ml) : 0;     // RoPE position
    const int slot_l = ml < p.M ? __ldg(p.row_slot + ml) : 0;   // cache slot
    const int sid_l = ml < p.M ? __ldg(p.row_stream + ml) : 0;
    float4 t[kRowsPerWarp];
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int pos = __shfl_sync(0xffffffffu, pos_l, warp + kEpiWarps * i);
        t[i] = region != 2 ? __ldg(reinterpret_cast<const float4*>(
                                 p.rope + (long long)min(max(pos, 0), p.rope_rows - 1) * kMaxPairs + (d >> 1)))
                           : make_float4(1.f, 0.f, 1.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int j = warp + kEpiWarps * i, m = mbase + j;
        const int pos = __shfl_sync(0xffffffffu, slot_l, j);
        const int sid = __shfl_sync(0xffffffffu, sid_l, j);
        const float4 a = *reinterpret_cast<const float4*>(st + j * kStageStride + 4 * lane);
        float x0 = a.x * sc.x, x1 = a.y * sc.y, x2 = a.z * sc.z, x3 = a.w * sc.w;
        if (region != 2) {
            const float y0 = __fsub_rn(__fmul_rn(x0, t[i].x), __fmul_rn(x1, t[i].y));
            const float y1 = __fadd_rn(__fmul_rn(x0, t[i].y), __fmul_rn(x1, t[i].x));
            const float y2 = __fsub_rn(__fmul_rn(x2, t[i].z), __fmul_rn(x3, t[i].w));
            const float y3 = __fadd_rn(__fmul_rn(x2, t[i].w), __fmul_rn(x3, t[i].z));
            x0 = y0;
            x1 = y1;
            x2 = y2;
            x3 = y3;
        }
        if (m >= p.M) continue;
        if (region == 0) {
            if (p.yq_hi) {
                x0 *= p.yq_scale;
                x1 *= p.yq_scale;
                x2 *= p.yq_scale;
                x3 *= p.yq_scale;
                const uint2 hi = make_uint2(pack_bf16x2(x0, x1), pack_bf16x2(x2, x3));
                const uint2 lo = make_uint2(pack_bf16x2(x0 - bf16lo(hi.x), x1 - bf16hi(hi.x)),
                                            pack_bf16x2(x2 - bf16lo(hi.y), x3 - bf16hi(hi.y)));
                *reinterpret_cast<uint2*>(p.yq_hi + (long long)m * hd + f) = hi;
                *reinterpret_cast<uint2*>(p.yq_lo + (long long)m * hd + f) = lo;
            } else {
                *reinterpret_cast<float4*>(p.yq + (long long)m * hd + f) = make_float4(x0, x1, x2, x3);
            }
            continue;
        }
        if (sid < 0 || sid >= p.num_streams || pos < 0 || pos >= p.capacity) {
            set_error(p.err, DEV_ERR_CAPACITY);
            continue;
        }
        const bool is_k = region == 1;
        const int kvh = (f - hd - (is_k ? 0 : kvd)) / kHeadDim;
        const uint2 packed = make_uint2(pack_bf16x2(x0, x1), pack_bf16x2(x2, x3));
        __nv_bfloat16* cache = is_k ? p.k_cache : p.v_cache;
        for (int rep = 0; rep < group; ++rep)
            *reinterpret_cast<uint2*>(cache + kv_offset(sid, pos, kvh * group + rep, p.num_streams, p.capacity) + d) =
                packed;
    }
}

// The other epilogues on the same staged layout (warp w rows w + 8i, lane l features
// n0 + 4l .. 4l + 3), with linear.cu's epilogue_pair arithmetic. EPI_RESID reads all its old
// values before its first store.
template <int EPI>
__device__ __forceinline__ void plain_rows(const LinearArgs& p, const float* st, int n0, int mbase, int z,
                                           int warp = threadIdx.x >> 5) {
    const int lane = threadIdx.x & 31;
    const int f = n0 + 4 * lane;
    const float4 sc = p.scale ? __ldg(reinterpret_cast<const float4*>(p.scale + f)) : make_float4(1.f, 1.f, 1.f, 1.f);
    float4 bias = make_float4(0.f, 0.f, 0.f, 0.f);
    if (EPI >= EPI_BIAS && p.bias) bias = __ldg(reinterpret_cast<const float4*>(p.bias + f));
    if (EPI == EPI_COND) {  // the step's time embedding joins the bias
        const float4 t = __ldg(reinterpret_cast<const float4*>(p.aux + f));
        bias = make_float4(bias.x + t.x, bias.y + t.y, bias.z + t.z, bias.w + t.w);
    }
    float4 old[kRowsPerWarp], gate[kRowsPerWarp];
    if (EPI == EPI_RESID || EPI == EPI_GATE_RESID) {
#pragma unroll
        for (int i = 0; i < kRowsPerWarp; ++i) {
            const int m = mbase + warp + kEpiWarps * i;
            const bool live = m < p.M;
            old[i] = live ? *reinterpret_cast<const float4*>(p.y + (long long)m * p.N + f) : make_float4(0.f, 0.f, 0.f, 0.f);
            if (EPI == EPI_GATE_RESID)
                gate[i] = live ? *reinterpret_cast<const float4*>(p.aux + (long long)m * p.aux_stride + f)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
#pragma unroll
    for (int i = 0; i < kRowsPerWarp; ++i) {
        const int j = warp + kEpiWarps * i, m = mbase + j;
        if (m >= p.M) break;
        const float4 a = *reinterpret_cast<const float4*>(st + j * kStageStride + 4 * lane);
        const float x0 = a.x * sc.x, x1 = a.y * sc.y, x2 = a.z * sc.z, x3 = a.w * sc.w;
        const long long at = (long long)m * p.N + f;
        if (EPI == EPI_F32) {
            *reinterpret_cast<float4*>(p.y + at) = make_float4(x0, x1, x2, x3);
        } else if (EPI == EPI_PARTIAL) {
            *reinterpret_cast<float4*>(p.y + (long long)z * p.M * p.N + at) = make_float4(x0, x1, x2, x3);
        } else if (EPI == EPI_RESID) {
            *reinterpret_cast<float4*>(p.y + at) =
                make_float4(old[i].x + x0, old[i].y + x1, old[i].z + x2, old[i].w + x3);
        } else if (EPI == EPI_BIAS) {
            *reinterpret_cast<float4*>(p.y + at) = make_float4(x0 + bias.x, x1 + bias.y, x2 + bias.z, x3 + bias.w);
        } else if (EPI == EPI_GATE_RESID) {  // x += gate * (W h + b)
            *reinterpret_cast<float4*>(p.y + at) =
                make_float4(old[i].x + gate[i].x * (x0 + bias.x), old[i].y + gate[i].y * (x1 + bias.y),
                            old[i].z + gate[i].z * (x2 + bias.z), old[i].w + gate[i].w * (x3 + bias.w));
        } else if (EPI == EPI_COND || EPI == EPI_BIAS_SILU) {  // bf16 hi/lo of silu(W x + b [+ t])
            uint2 hi, lo;
            const float y0 = silu(x0 + bias.x), y1 = silu(x1 + bias.y), y2 = silu(x2 + bias.z), y3 = silu(x3 + bias.w);
            hi.x = pack_bf16x2(y0, y1);
            hi.y = pack_bf16x2(y2, y3);
            lo.x = pack_bf16x2(y0 - bf16lo(hi.x), y1 - bf16hi(hi.x));
            lo.y = pack_bf16x2(y2 - bf16lo(hi.y), y3 - bf16hi(hi.y));
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.yb) + at) = hi;
            *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(p.yb_lo) + at) = lo;
        } else {  // EPI_GELU: f16 hi/lo planes
            uint2 hi, lo;
            split_f16x2(gelu_tc(x0, p.gelu_tanh), gelu_tc(x1, p.gelu_tanh), hi.x, lo.x);
            split_f16x2(gelu_tc(x2, p.gelu_tanh), gelu_tc(x3, p.gelu_tanh), hi.y, lo.y);
            *reinterpret_cast<uint2*>(static_cast<__half*>(p.yb) + at) = hi;
            *reinterpret_cast<uint2*>(static_cast<__half*>(p.yb_lo) + at) = lo;
        }
    }
}

// The epilogue of a 128-feature x RT-row tile (all 16 warps; the ring at `smem` is drained):
// warp w reads TMEM lane quarter w % 4, columns (rows) c + 8 (w / 4) .. + 7 of each 32-row chunk,
// and transposes them through shared memory, so that lanes then own feature quads and store 16
// bytes per row (qkv_rows / plain_rows).
template <int EPI, int RT>
__device__ __forceinline__ void drain_tile(const LinearArgs& p, unsigned char* smem, uint32_t tmem, int n0,
                                           int m0, int z, bool got, bool lo_cols) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncwarp();  // tcgen05.ld below is warp-collective
    tc_fence_after();
#pragma unroll 1
    for (int c = 0; c < RT; c += 32) {
        constexpr int CW = 32 / (kEpiWarps / 4);  // columns (rows) per warp
        const int quarter = warp & 3, part = warp >> 2;
        float v[CW];
        const uint32_t col = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(c + CW * part);
        tmem_ld<CW>(col, v);
        if (lo_cols) {  // the lo plane's products of the same rows, RT columns further
            float w[CW];
            tmem_ld<CW>(col + RT, w);
#pragma unroll
            for (int j = 0; j < CW; ++j) v[j] += w[j];
        }
        float* st = reinterpret_cast<float*>(smem);
        __syncthreads();  // the previous chunk's readers are done
#pragma unroll
        for (int j = 0; j < CW; ++j) st[(CW * part + j) * kStageStride + 32 * quarter + lane] = v[j];
        __syncthreads();
        if (got) {
            if (EPI == EPI_QKV) qkv_rows(p, st, n0, m0 + c);
            else plain_rows<EPI>(p, st, n0, m0 + c, z);
        }
    }
}

template <int EPI, int RT, int WM>
__global__ void __launch_bounds__(kThreadsTma) linear_tma_kernel(const __grid_constant__ LinearArgs p,
                                                                 const __grid_constant__ CUtensorMap tm_w,
                                                                 const __grid_constant__ CUtensorMap tm_wlo,
                                                                 const __grid_constant__ CUtensorMap tm_x,
                                                                 const __grid_constant__ CUtensorMap tm_xlo) {
    using T = TmaTile<RT, WM>;
    constexpr int S = T::kStages;
    constexpr bool W8 = WM == kW8, WLO = WM == kW16Lo;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + T::kBarOffset);  // a stage's weights landed
    uint64_t* xfull = wfull + S;                                           // its activations landed
    uint64_t* conv = xfull + S;                                            // kW8: its weights widened
    uint64_t* empty = conv + S;                                            // its MMAs are done
    uint64_t* done = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int s_w_issued, s_issued, s_consumed;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * FT, m0 = blockIdx.y * RT, z = blockIdx.z;
    const int k_len = p.K / p.splits;
    const int k0 = z * k_len;
    const int KT = k_len / KS;
    const bool has_lo = p.a_lo != nullptr;
    const uint32_t x_tx = (has_lo ? 2u : 1u) * T::kXBytes;
    const bool converter = W8 && warp >= 4 && warp < 4 + kConvWarps;  // warps 4..11

    if (tid == 0) {
        s_w_issued = 0;
        s_issued = 0;
        s_consumed = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&wfull[s], 1);
            mbar_init(&xfull[s], 1);
            mbar_init(&conv[s], kConvWarps);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(T::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (tid == 0) stamp_mark(p.stamps, p.stamp, STAMP_ENTRY);
    if (tid == 0) {
        // ---- TMA producer ----------------------------------------------------------------------
        const uint64_t pol_w = policy_evict_last();  // weights: reread every frame
        auto load_w = [&](int kt, uint32_t sa, int st) {
            mbar_arrive_expect_tx(&wfull[st], T::kWTx);
            // kW8: the int8 tile goes to the upper half of the slot, where the converters find it.
            tma_load_2d_hint(sa + (W8 ? FT * KS : 0), &tm_w, k0 + kt * KS, n0, &wfull[st], pol_w);
            if (WLO) tma_load_2d_hint(sa + T::kWBytes, &tm_wlo, k0 + kt * KS, n0, &wfull[st], pol_w);
            s_w_issued = kt + 1;
        };
        const int pre = KT < S ? KT : S;
        for (int kt = 0; kt < pre; ++kt) load_w(kt, base + kt * T::kStageBytes, kt);
        grid_dep_wait();
        stamp_mark(p.stamps, p.stamp, STAMP_START);
        for (int kt = 0; kt < KT; ++kt) {
            const int st = kt % S;
            const uint32_t sa = base + st * T::kStageBytes;
            if (kt >= pre) {
                if (!mbar_wait(&empty[st], ((kt / S) & 1) ^ 1)) {
                    set_error(p.err, DEV_ERR_TIMEOUT);
                    break;
                }
                load_w(kt, sa, st);
            }
            mbar_arrive_expect_tx(&xfull[st], x_tx);
            tma_load_2d(sa + T::kXOffset, &tm_x, k0 + kt * KS, m0, &xfull[st]);
            if (has_lo) tma_load_2d(sa + T::kXOffset + T::kXBytes, &tm_xlo, k0 + kt * KS, m0, &xfull[st]);
            s_issued = kt + 1;
        }
    } else if (converter) {
        // ---- kW8 converters: weights need no predecessor, so they start at once -----------------
        const int t = tid - 128;
        for (int kt = 0; kt < KT; ++kt) {
            const int st = kt % S;
            const bool landed = mbar_wait(&wfull[st], (kt / S) & 1);
            const bool ok = p.a_f16 ? widen_w8<true>(smem + st * T::kStageBytes, t, landed)
                                    : widen_w8<false>(smem + st * T::kStageBytes, t, landed);
            if (!ok) {
                set_error(p.err, DEV_ERR_TIMEOUT);
                break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv[st]);
        }
        grid_dep_wait();  // the epilogue below reads what predecessors wrote
    } else {
        grid_dep_wait();
        if (tid == 32) {
            // ---- MMA issuer --------------------------------------------------------------------
            // The X hi and lo tiles lie back to back in the stage (RT rows each, 1024-byte
            // aligned), so with a lo plane one MMA of N = 2 RT takes both: the weight tile is
            // read once per k step instead of once per plane. Columns RT.. hold the lo rows.
            const uint32_t idesc1 = p.a_f16 ? idesc_f16<RT>() : idesc_bf16<RT>();
            const uint32_t idesc2 = p.a_f16 ? idesc_f16<2 * RT>() : idesc_bf16<2 * RT>();
            const uint32_t idesc = has_lo ? idesc2 : idesc1;
            for (int kt = 0; kt < KT; ++kt) {
                const int st = kt % S;
                const uint32_t ph = (kt / S) & 1;
                if (!mbar_wait(W8 ? &conv[st] : &wfull[st], ph) || !mbar_wait(&xfull[st], ph)) {
                    set_error(p.err, DEV_ERR_TIMEOUT);
                    break;
                }
                tc_fence_after();
                const uint32_t sa = base + st * T::kStageBytes;
                const uint64_t dw = sw128_desc(sa), dwl = sw128_desc(sa + T::kWBytes);
                const uint64_t dx = sw128_desc(sa + T::kXOffset);
#pragma unroll
                for (int kk = 0; kk < KS / 16; ++kk) {  // 32 bytes of K per MMA
                    tc_mma(tmem, dw + 2 * kk, dx + 2 * kk, idesc, (kt | kk) ? 1u : 0u);
                    if (WLO) tc_mma(tmem, dwl + 2 * kk, dx + 2 * kk, idesc1, 1u);  // into the hi columns
                }
                tc_commit(&empty[st]);
                s_consumed = kt + 1;
            }
            tc_commit(done);  // arrives once every MMA issued above has completed
        }
    }
    __syncwarp();

    // ---- epilogue: feature n0 + 32w + lane, rows m0 .. m0 + RT - 1 ------------------------------
    const bool got = mbar_wait(done, 0);
    if (!got) set_error(p.err, DEV_ERR_TIMEOUT);
    // The next kernel may launch now: its CTAs take SM room only while this epilogue runs, not
    // through the whole pipeline (room a concurrent lane's kernels can use).
    if (tid == 0) grid_dep_launch();
    drain_tile<EPI, RT>(p, smem, tmem, n0, m0, z, got, has_lo);

    if (tid == 0) stamp_mark(p.stamps, p.stamp, STAMP_END);
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        // Copies issued but never consumed (only after a timeout): let them land before exit.
        for (int kt = s_consumed; kt < s_w_issued; ++kt) mbar_wait(&wfull[kt % S], (kt / S) & 1);
        for (int kt = s_consumed; kt < s_issued; ++kt) mbar_wait(&xfull[kt % S], (kt / S) & 1);
    }
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(T::kTmemCols)
                     : "memory");
    }
}

// ---- decode-size linears on int8 weights, widened into tensor memory ----------------------------
//
// linear_i8_kernel: the kW8 form of linear_tma_kernel (one 128-feature x RT-row tile per CTA,
// 512 threads, the same MMAs and epilogues) with the widened weights in tensor memory: the MMA
// takes its A operand (the 128 x 16 weight slice of a k step) from TMEM, so neither the widening
// nor the MMA's weight reads touch shared memory, and a stage in shared memory is only the int8
// tile (8 KB) and the activation tiles (hi, lo).
//   thread 0:     TMA producer; the int8 tiles of the first stages before the wait on the
//                 predecessor grid (weights never change), the activation tiles after it.
//   warps 4..11:  converters. Warp w takes TMEM lane quarter w % 4 (its rows: 32 (w % 4) + lane)
//                 and half (w - 4) / 4 of the stage's 64 k: it reads the row's 32 int8 weights,
//                 widens them in registers and stores them as 16 packed 16-bit pairs into the
//                 stage's A slot (tcgen05.st), then waits for the stores (tcgen05.wait::st).
//   thread 32:    MMA issuer, A from TMEM (lane = feature row, column c = k 2c, 2c + 1), B the
//                 activation tile in shared memory.
// The int8 tile is copied with the 64-byte swizzle (16-byte chunk c of row r at c ^ ((r / 2) % 4)),
// so a quarter-warp's reads of 8 rows hit the eight distinct bank groups.
//
// TMEM: the accumulator (2 RT columns) and kStages A slots of 32 columns, 256 columns per CTA.
// Shared memory (5 stages, 81 KB) keeps at most two CTAs of this kernel on an SM, so CTAs that
// share an SM never ask for more than the SM's 512 columns (an allocation never waits, which could
// otherwise deadlock against an early-launched successor holding TMEM while it waits on us).
template <int RT>
struct I8Tile {
    static constexpr int kStages = 5;
    static constexpr int kQ8Stages = 3;           // q8_0 form: a hi and a lo A slot per stage
    static constexpr int kW8Bytes = FT * KS;      // int8 tile
    static constexpr int kXBytes = RT * KS * 2;   // one activation plane
    static constexpr int kStageBytes = kW8Bytes + 2 * kXBytes;
    static constexpr int kXOffset = kW8Bytes;
    static constexpr int kBarOffset = kStages * kStageBytes;
    static constexpr int kSmem = 1024 + kBarOffset + 256;
    static constexpr uint32_t kAccCols = 2 * RT;
    static constexpr uint32_t kACols = KS / 2;    // one stage's A slot: 64 k as 32 packed pairs
    static constexpr uint32_t kTmemCols = 256;
    static_assert(kAccCols + kStages * kACols <= kTmemCols, "accumulator and A slots fit");
    static_assert(kAccCols + kQ8Stages * 2 * kACols <= kTmemCols, "q8_0: accumulator and hi/lo A slots fit");
    static_assert(kStageBytes % 1024 == 0 && kXBytes % 1024 == 0, "swizzled tiles stay 1024-byte aligned");
    static_assert(32 * (FT + 4) * 4 <= kBarOffset, "the epilogue's staging tile fits");
    static_assert(3 * (kSmem + 1024) > 228 * 1024, "at most two CTAs per SM (TMEM: 2 x 256 columns)");
    static_assert((4 * kStages + 1) * 8 + 4 <= 256, "barriers fit the tail");
};

// D (TMEM) += A (TMEM) x B (smem), or D = A x B when accumulate is 0.
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 16 consecutive TMEM columns of this warp's 32 lanes from registers (tcgen05.st.32x32b.x16).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// 8 consecutive TMEM columns of this warp's 32 lanes from registers (tcgen05.st.32x32b.x8).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

template <int EPI, int RT, bool Q8>
__global__ void __launch_bounds__(kThreadsTma) linear_i8_kernel(const __grid_constant__ LinearArgs p,
                                                                const __grid_constant__ CUtensorMap tm_w,
                                                                const __grid_constant__ CUtensorMap tm_x,
                                                                const __grid_constant__ CUtensorMap tm_xlo) {
    using T = I8Tile<RT>;
    // q8_0 form (Q8, p.wblk): 3 stages, each with a hi and a lo A slot; else 5 with one.
    constexpr int S = Q8 ? T::kQ8Stages : T::kStages;
    constexpr uint32_t slot_cols = Q8 ? 2 * T::kACols : T::kACols;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + T::kBarOffset);  // int8 tile landed
    uint64_t* xfull = wfull + S;                                           // activations landed
    uint64_t* conv = xfull + S;                                            // A slot written
    uint64_t* empty = conv + S;                                            // the stage's MMAs done
    uint64_t* done = empty + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    __shared__ int s_w_issued, s_issued, s_consumed;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * FT, m0 = blockIdx.y * RT, z = blockIdx.z;
    const int k_len = p.K / p.splits;
    const int k0 = z * k_len;
    const int KT = k_len / KS;
    const bool has_lo = p.a_lo != nullptr;
    const uint32_t x_tx = (has_lo ? 2u : 1u) * T::kXBytes;

    if (tid == 0) {
        s_w_issued = 0;
        s_issued = 0;
        s_consumed = 0;
        for (int i = 0; i < S; ++i) {
            mbar_init(&wfull[i], 1);
            mbar_init(&xfull[i], 1);
            mbar_init(&conv[i], kConvWarps);
            mbar_init(&empty[i], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(T::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tmem_a = tmem + T::kAccCols;  // A slot(s) of stage s: + s * slot_cols columns

    if (tid == 0) stamp_mark(p.stamps, p.stamp, STAMP_ENTRY);
    if (tid == 0) {
        // ---- TMA producer ----------------------------------------------------------------------
        const uint64_t pol_w = policy_evict_last();  // weights: reread every frame
        const int pre = KT < S ? KT : S;
        for (int kt = 0; kt < pre; ++kt) {
            mbar_arrive_expect_tx(&wfull[kt], T::kW8Bytes);
            tma_load_2d_hint(base + kt * T::kStageBytes, &tm_w, k0 + kt * KS, n0, &wfull[kt], pol_w);
            s_w_issued = kt + 1;
        }
        grid_dep_wait();
        stamp_mark(p.stamps, p.stamp, STAMP_START);
        for (int kt = 0; kt < KT; ++kt) {
            const int st = kt % S;
            const uint32_t sa = base + st * T::kStageBytes;
            if (kt >= pre) {
                if (!mbar_wait(&empty[st], ((kt / S) & 1) ^ 1)) {
                    set_error(p.err, DEV_ERR_TIMEOUT);
                    break;
                }
                mbar_arrive_expect_tx(&wfull[st], T::kW8Bytes);
                tma_load_2d_hint(sa, &tm_w, k0 + kt * KS, n0, &wfull[st], pol_w);
                s_w_issued = kt + 1;
            }
            mbar_arrive_expect_tx(&xfull[st], x_tx);
            tma_load_2d(sa + T::kXOffset, &tm_x, k0 + kt * KS, m0, &xfull[st]);
            if (has_lo) tma_load_2d(sa + T::kXOffset + T::kXBytes, &tm_xlo, k0 + kt * KS, m0, &xfull[st]);
            s_issued = kt + 1;
        }
    } else if (warp >= 4 && warp < 4 + kConvWarps) {
        // ---- converters: int8 row -> 16-bit pairs in the stage's A slot --------------------------
        const int quarter = warp & 3, half = (warp - 4) >> 2;
        const int r = 32 * quarter + lane;  // this thread's weight row (TMEM lane)
        const uint32_t lane_base = (uint32_t)(32 * quarter) << 16;
        for (int kt = 0; kt < KT; ++kt) {
            const int st = kt % S;
            const bool landed = mbar_wait(&wfull[st], (kt / S) & 1);
            if (__any_sync(0xffffffffu, !landed)) {  // the whole warp leaves together
                set_error(p.err, DEV_ERR_TIMEOUT);
                break;
            }
            const unsigned char* row = smem + st * T::kStageBytes + r * KS;
            if constexpr (Q8) {
                // hi = RN16(q d) and lo = RN16(q d - hi) in f16 arithmetic: q and d (the block
                // scale over the row's power of two, an exact f16) are exact, the product is
                // rounded once (mul) and the residual once (fma), subnormals kept: the layer's
                // own f16 planes, bit for bit. This thread's 32 weights are one q8_0 block
                // (k 32 half .. of the stage), stored 16 k at a time (the kernel stays within
                // 56 registers a thread, so that a CTA still fits beside the decode attention's
                // on an SM: each quarter of the register file holds four of these warps and up
                // to three of the attention's).
                const __half d = p.wblk[(size_t)(n0 + r) * (p.K / 32) + (k0 + kt * KS) / 32 + half];
                const __half2 d2 = __halves2half2(d, d);
                const uint32_t at = tmem_a + lane_base + (uint32_t)st * slot_cols + 16 * half;
#pragma unroll
                for (int c2 = 0; c2 < 2; ++c2) {
                    const int c = 2 * half + c2;
                    const uint4 q = *reinterpret_cast<const uint4*>(row + ((c ^ ((r >> 1) & 3)) << 4));
                    uint32_t hv[8], lv[8];
                    i8x4_to_f16x4(q.x, hv[0], hv[1]);
                    i8x4_to_f16x4(q.y, hv[2], hv[3]);
                    i8x4_to_f16x4(q.z, hv[4], hv[5]);
                    i8x4_to_f16x4(q.w, hv[6], hv[7]);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const __half2 qj = *reinterpret_cast<const __half2*>(&hv[j]);
                        const __half2 h = __hmul2(qj, d2);
                        const __half2 l = __hfma2(qj, d2, __hneg2(h));
                        hv[j] = *reinterpret_cast<const uint32_t*>(&h);
                        lv[j] = *reinterpret_cast<const uint32_t*>(&l);
                    }
                    tmem_st8(at + 8 * c2, hv);
                    tmem_st8(at + T::kACols + 8 * c2, lv);
                }
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&conv[st]);
                continue;
            }
            uint32_t v[16];
#pragma unroll
            for (int c2 = 0; c2 < 2; ++c2) {  // 16-byte chunks 2 half + c2 (k 16 (2 half + c2) ..)
                const int c = 2 * half + c2;
                const uint4 q = *reinterpret_cast<const uint4*>(row + ((c ^ ((r >> 1) & 3)) << 4));
                if (p.a_f16) {
                    i8x4_convert<true>(q.x, v[8 * c2 + 0], v[8 * c2 + 1]);
                    i8x4_convert<true>(q.y, v[8 * c2 + 2], v[8 * c2 + 3]);
                    i8x4_convert<true>(q.z, v[8 * c2 + 4], v[8 * c2 + 5]);
                    i8x4_convert<true>(q.w, v[8 * c2 + 6], v[8 * c2 + 7]);
                } else {
                    i8x4_convert<false>(q.x, v[8 * c2 + 0], v[8 * c2 + 1]);
                    i8x4_convert<false>(q.y, v[8 * c2 + 2], v[8 * c2 + 3]);
                    i8x4_convert<false>(q.z, v[8 * c2 + 4], v[8 * c2 + 5]);
                    i8x4_convert<false>(q.w, v[8 * c2 + 6], v[8 * c2 + 7]);
                }
            }
            tmem_st16(tmem_a + lane_base + (uint32_t)st * slot_cols + 16 * half, v);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&conv[st]);
        }
    } else if (tid == 32) {
        // ---- MMA issuer --------------------------------------------------------------------
        const uint32_t idesc1 = p.a_f16 ? idesc_f16<RT>() : idesc_bf16<RT>();
        const uint32_t idesc2 = p.a_f16 ? idesc_f16<2 * RT>() : idesc_bf16<2 * RT>();
        const uint32_t idesc = has_lo ? idesc2 : idesc1;
        for (int kt = 0; kt < KT; ++kt) {
            const int st = kt % S;
            const uint32_t ph = (kt / S) & 1;
            if (!mbar_wait(&conv[st], ph) || !mbar_wait(&xfull[st], ph)) {
                set_error(p.err, DEV_ERR_TIMEOUT);
                break;
            }
            tc_fence_after();
            const uint64_t dx = sw128_desc(base + st * T::kStageBytes + T::kXOffset);
            const uint32_t a = tmem_a + (uint32_t)st * slot_cols;
#pragma unroll
            for (int kk = 0; kk < KS / 16; ++kk) {  // 16 k per MMA: 8 A columns, 32 bytes of B
                tc_mma_ts(tmem, a + 8 * kk, dx + 2 * kk, idesc, (kt | kk) ? 1u : 0u);
                // q8_0: the weights' lo plane times the activations' hi rows (the first RT rows
                // of the stage's B tile; lo x lo is below the products' f32 rounding).
                if (Q8) tc_mma_ts(tmem, a + T::kACols + 8 * kk, dx + 2 * kk, idesc1, 1u);
            }
            tc_commit(&empty[st]);
            s_consumed = kt + 1;
        }
        tc_commit(done);  // arrives once every MMA issued above has completed
    }
    grid_dep_wait();  // the epilogue reads what predecessors wrote (a no-op once passed)
    __syncwarp();

    const bool got = mbar_wait(done, 0);
    if (!got) set_error(p.err, DEV_ERR_TIMEOUT);
    if (tid == 0) grid_dep_launch();
    drain_tile<EPI, RT>(p, smem, tmem, n0, m0, z, got, has_lo);

    if (tid == 0) stamp_mark(p.stamps, p.stamp, STAMP_END);
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        // Copies issued but never consumed (only after a timeout): let them land before exit.
        for (int kt = s_consumed; kt < s_w_issued; ++kt) mbar_wait(&wfull[kt % S], (kt / S) & 1);
        for (int kt = s_consumed; kt < s_issued; ++kt) mbar_wait(&xfull[kt % S], (kt / S) & 1);
    }
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(T::kTmemCols)
                     : "memory");
    }
}

// ---- persistent prompt-size linears ----------------------------------------------------------
//
// One CTA per SM walks 128-feature x 128-row tiles (tile t = blockIdx.x + i * gridDim.x,
// feature tile t % NT, row tile t / NT) with two TMEM accumulators, so the epilogue of one tile
// runs while the next tile's loads and MMAs do:
//   warp 0, lane 0: TMA producer over a 4-stage (3 with a weight lo plane) ring of
//                   {W 128x64 (+ lo), X hi 128x64, X lo}, weights and activations on separate
//                   barriers
//   warp 1, lane 0: MMA issuer, tcgen05.commit frees each stage and fills an accumulator
//   warps 2..17:    epilogue, two accumulators in turn: 4 x 32-row chunks through a staging
//                   tile (warp w reads TMEM lane quarter w % 4, 8 columns), then the same
//                   row epilogues as linear_tma_kernel (2 rows per warp and chunk)
//   warps 18..25:   kW8 only: the converters (widen_w8), one stage after another (the layer
//                   stack widens a prompt's weights once per call instead, see abi.cu)
// Every wait is bounded; a timed-out wait sets DEV_ERR_TIMEOUT and a shared abort flag that
// ends every role's loop.
constexpr int PT = 128;   // rows per tile (MMA N)

template <int WM>
struct PersistTile {
    static constexpr int PS = WM == kW16Lo ? 3 : 4;  // ring stages: 192 KB either way
    static constexpr int kWBytes = FT * KS * 2;
    static constexpr int kXBytes = PT * KS * 2;
    static constexpr int kStageBytes = (WM == kW16Lo ? 2 : 1) * kWBytes + 2 * kXBytes;
    static constexpr int kXOffset = (WM == kW16Lo ? 2 : 1) * kWBytes;
    static constexpr int kStageOffset = PS * kStageBytes;              // the epilogue's staging tile
    static constexpr int kBarOffset = kStageOffset + 32 * kStageStride * 4;
    static constexpr int kSmem = 1024 + kBarOffset + 256;
    static constexpr uint32_t kWTx = WM == kW8 ? FT * KS : (WM == kW16Lo ? 2 : 1) * kWBytes;
    static constexpr int kConvWarp0 = 2 + kEpiWarps;
    static constexpr int kWarps = kConvWarp0 + (WM == kW8 ? kConvWarps : 0);
    static constexpr int kThreads = 32 * kWarps;
    static_assert(kStageBytes % 1024 == 0, "stages stay 1024-byte aligned");
    static_assert(kSmem <= 227 * 1024, "fits one CTA per SM");
    static_assert(4 * PS * 8 + 4 * 8 + 4 <= 256, "barriers fit the tail");
};

__device__ __forceinline__ void epi_bar_sync() {  // the 16 epilogue warps only
    asm volatile("bar.sync 1, %0;" ::"r"(32 * kEpiWarps) : "memory");
}
// The same barrier, returning whether `v` held in any epilogue thread (one answer for all).
__device__ __forceinline__ bool epi_bar_any(bool v) { return bar_any<1, 32 * kEpiWarps>(v); }

template <int EPI, int WM>
__global__ void __launch_bounds__(PersistTile<WM>::kThreads, 1) linear_persist_kernel(
    const __grid_constant__ LinearArgs p, const __grid_constant__ CUtensorMap tm_w,
    const __grid_constant__ CUtensorMap tm_wlo, const __grid_constant__ CUtensorMap tm_x,
    const __grid_constant__ CUtensorMap tm_xlo) {
    using T = PersistTile<WM>;
    constexpr int PS = T::PS;
    constexpr bool W8 = WM == kW8, WLO = WM == kW16Lo;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    uint64_t* wfull = reinterpret_cast<uint64_t*>(smem + T::kBarOffset);
    uint64_t* xfull = wfull + PS;
    uint64_t* conv = xfull + PS;
    uint64_t* empty = conv + PS;
    uint64_t* acc_full = empty + PS;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    __shared__ int s_abort, s_issued, s_consumed;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NT = p.N / FT, MT = (p.M + PT - 1) / PT, tiles = NT * MT, KT = p.K / KS;
    const bool has_lo = p.a_lo != nullptr;
    const uint32_t x_tx = (has_lo ? 2u : 1u) * T::kXBytes;

    if (tid == 0) {
        s_abort = 0;
        s_issued = 0;
        s_consumed = 0;
        for (int i = 0; i < PS; ++i) {
            mbar_init(&wfull[i], 1);
            mbar_init(&xfull[i], 1);
            mbar_init(&conv[i], kConvWarps);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiWarps);
        }
        fence_mbar_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * PT)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tid == 0) stamp_mark(p.stamps, p.stamp, STAMP_ENTRY);
    auto fail = [&]() {
        set_error(p.err, DEV_ERR_TIMEOUT);
        atomicExch(&s_abort, 1);
    };
    auto aborted = [&]() { return *reinterpret_cast<volatile int*>(&s_abort) != 0; };

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ------------------------------------------------------------------
            const uint64_t pol_w = policy_evict_last();
            grid_dep_wait();
            stamp_mark(p.stamps, p.stamp, STAMP_START);
            int kk = 0;
            for (int t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x) {
                const int n0 = (t % NT) * FT, m0 = (t / NT) * PT;
                for (int kt = 0; kt < KT; ++kt, ++kk) {
                    const int st = kk % PS;
                    if (kk >= PS && !mbar_wait(&empty[st], ((kk / PS) & 1) ^ 1)) {
                        fail();
                        break;
                    }
                    const uint32_t sa = base + st * T::kStageBytes;
                    mbar_arrive_expect_tx(&wfull[st], T::kWTx);
                    tma_load_2d_hint(sa + (W8 ? FT * KS : 0), &tm_w, kt * KS, n0, &wfull[st], pol_w);
                    if (WLO) tma_load_2d_hint(sa + T::kWBytes, &tm_wlo, kt * KS, n0, &wfull[st], pol_w);
                    mbar_arrive_expect_tx(&xfull[st], x_tx);
                    tma_load_2d(sa + T::kXOffset, &tm_x, kt * KS, m0, &xfull[st]);
                    if (has_lo) tma_load_2d(sa + T::kXOffset + T::kXBytes, &tm_xlo, kt * KS, m0, &xfull[st]);
                    s_issued = kk + 1;
                }
            }
            grid_dep_launch();
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer --------------------------------------------------------------------
            const uint32_t idesc = p.a_f16 ? idesc_f16<PT>() : idesc_bf16<PT>();
            int kk = 0, i = 0;
            for (int t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x, ++i) {
                const int acc = i & 1, use = i >> 1;
                if (use > 0 && !mbar_wait(&acc_empty[acc], (use - 1) & 1)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * PT);
                bool ok = true;
                for (int kt = 0; kt < KT; ++kt, ++kk) {
                    const int st = kk % PS;
                    const uint32_t ph = (kk / PS) & 1;
                    if (!mbar_wait(W8 ? &conv[st] : &wfull[st], ph) || !mbar_wait(&xfull[st], ph)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = base + st * T::kStageBytes;
                    const uint64_t dw = sw128_desc(sa), dwl = sw128_desc(sa + T::kWBytes);
                    const uint64_t dx = sw128_desc(sa + T::kXOffset), dxl = sw128_desc(sa + T::kXOffset + T::kXBytes);
#pragma unroll
                    for (int k2 = 0; k2 < KS / 16; ++k2) {
                        tc_mma(d, dw + 2 * k2, dx + 2 * k2, idesc, (kt | k2) ? 1u : 0u);
                        if (has_lo) tc_mma(d, dw + 2 * k2, dxl + 2 * k2, idesc, 1u);
                        if (WLO) tc_mma(d, dwl + 2 * k2, dx + 2 * k2, idesc, 1u);
                    }
                    tc_commit(&empty[st]);
                    s_consumed = kk + 1;
                }
                if (!ok) {
                    fail();
                    break;
                }
                tc_commit(&acc_full[acc]);
            }
        }
    } else if (warp >= T::kConvWarp0) {
        // ---- kW8 converters -------------------------------------------------------------------
        const int cv = tid - 32 * T::kConvWarp0;
        int kk = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
            for (int kt = 0; kt < KT; ++kt, ++kk) {
                const int st = kk % PS;
                // Leave together on a timeout or an abort elsewhere (one answer for all).
                const bool landed = !aborted() && mbar_wait(&wfull[st], (kk / PS) & 1);
                ok = p.a_f16 ? widen_w8<true>(smem + st * T::kStageBytes, cv, landed)
                             : widen_w8<false>(smem + st * T::kStageBytes, cv, landed);
                if (!ok) {
                    fail();
                    break;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&conv[st]);
            }
        }
    } else {
        // ---- epilogue ------------------------------------------------------------------------
        grid_dep_wait();  // the residual epilogues read what predecessors wrote
        const int ew = warp - 2, quarter = warp & 3, part = ew >> 2;
        float* stg = reinterpret_cast<float*>(smem + T::kStageOffset);
        int i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
            const int acc = i & 1, use = i >> 1;
            const int n0 = (t % NT) * FT, m0 = (t / NT) * PT;
            const bool got = !aborted() && mbar_wait(&acc_full[acc], use & 1);
            if (!got) fail();
            if (epi_bar_any(!got)) break;  // every epilogue warp leaves together
            __syncwarp();
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < PT; c += 32) {
                float v[8];
                tmem_ld8(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(acc * PT + c + 8 * part), v);
                epi_bar_sync();  // the previous chunk's readers are done with the staging tile
#pragma unroll
                for (int j = 0; j < 8; ++j) stg[(8 * part + j) * kStageStride + 32 * quarter + lane] = v[j];
                epi_bar_sync();
                if (EPI == EPI_QKV) qkv_rows(p, stg, n0, m0 + c, ew);
                else plain_rows<EPI>(p, stg, n0, m0 + c, 0, ew);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        if (tid == 64) stamp_mark(p.stamps, p.stamp, STAMP_END);
    }

    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        // Copies issued but never consumed (only after a timeout): let them land before exit.
        for (int kk = s_consumed; kk < s_issued; ++kk) {
            mbar_wait(&wfull[kk % PS], (kk / PS) & 1);
            mbar_wait(&xfull[kk % PS], (kk / PS) & 1);
        }
    }
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * PT) : "memory");
    }
}

// linear_rows_kernel: the prompt-size linears with the operands' roles swapped. A is a tile of 128
// activation rows (hi and lo planes, two MMAs), B 256 weight features (MMA N = 256), so an
// accumulator is 128 rows (TMEM lanes) x 256 features (columns) and each activation byte that
// crosses from L2 feeds twice the features of linear_persist_kernel's 128-feature tiles:
// 64 KB per stage for 8.4 MFLOP against 48 KB for 4.2. Same roles and barriers otherwise:
//   warp 0, lane 0: TMA producer (3 stages of X hi, X lo and W; 2 with a weight lo plane)
//   warp 1, lane 0: MMA issuer into two 256-column accumulators (all 512 TMEM columns)
//   warps 2..17:    epilogue, per 32-row x 128-feature chunk: the four warps of the chunk's TMEM
//                   lane quarter read 32 columns each into the staging tile, then all 16 run the
//                   row epilogues of linear_tma_kernel on it (2 rows per warp)
// N must be a multiple of 256 and the weights 16-bit (planes or the widened prompt copy).
constexpr int NT2 = 256;  // features per tile (MMA N)

template <int WM>
struct RowsTile {
    static constexpr bool WLO = WM == kW16Lo;
    static constexpr int PS = WLO ? 2 : 3;             // ring stages: 192 KB either way
    static constexpr int kXBytes = PT * KS * 2;         // one activation plane: 16 KB
    static constexpr int kWBytes = NT2 * KS * 2;        // one weight plane: 32 KB
    static constexpr int kWOffset = 2 * kXBytes;
    static constexpr int kStageBytes = 2 * kXBytes + (WLO ? 2 : 1) * kWBytes;
    static constexpr int kStageOffset = PS * kStageBytes;  // the epilogue's staging tile
    static constexpr int kBarOffset = kStageOffset + 32 * kStageStride * 4;
    static constexpr int kSmem = 1024 + kBarOffset + 256;
    static constexpr int kThreads = 32 * (2 + kEpiWarps);
    static_assert(kStageBytes % 1024 == 0, "stages stay 1024-byte aligned");
    static_assert(kSmem <= 227 * 1024, "fits one CTA per SM");
    static_assert(3 * PS * 8 + 4 * 8 + 4 <= 256, "barriers fit the tail");
};

// 32 consecutive TMEM columns of this warp's 32 lanes (tcgen05.ld.32x32b.x32), one wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <int EPI, int WM>
__global__ void __launch_bounds__(RowsTile<WM>::kThreads, 1) linear_rows_kernel(
    const __grid_constant__ LinearArgs p, const __grid_constant__ CUtensorMap tm_w,
    const __grid_constant__ CUtensorMap tm_wlo, const __grid_constant__ CUtensorMap tm_x,
    const __grid_constant__ CUtensorMap tm_xlo) {
    using T = RowsTile<WM>;
    constexpr int PS = T::PS;
    constexpr bool WLO = T::WLO;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* smem = smem_raw + (base - raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + T::kBarOffset);  // a stage landed
    uint64_t* empty = full + PS;                                         // its MMAs are done
    uint64_t* acc_full = empty + PS;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    __shared__ int s_abort, s_issued, s_consumed;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NT = p.N / NT2, MT = (p.M + PT - 1) / PT, tiles = NT * MT, KT = p.K / KS;
    const bool has_lo = p.a_lo != nullptr;
    const uint32_t tx = (has_lo ? 2u : 1u) * T::kXBytes + (WLO ? 2u : 1u) * T::kWBytes;

    if (tid == 0) {
        s_abort = 0;
        s_issued = 0;
        s_consumed = 0;
        for (int i = 0; i < PS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kEpiWarps);
        }
        fence_mbar_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x)) : "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * NT2)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (tid == 0) stamp_mark(p.stamps, p.stamp, STAMP_ENTRY);
    auto fail = [&]() {
        set_error(p.err, DEV_ERR_TIMEOUT);
        atomicExch(&s_abort, 1);
    };
    auto aborted = [&]() { return *reinterpret_cast<volatile int*>(&s_abort) != 0; };

    if (warp == 0) {
        if (lane == 0) {
            // ---- TMA producer ------------------------------------------------------------------
            const uint64_t pol_w = policy_evict_last();
            grid_dep_wait();
            stamp_mark(p.stamps, p.stamp, STAMP_START);
            int kk = 0;
            for (int t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x) {
                const int n0 = (t % NT) * NT2, m0 = (t / NT) * PT;
                for (int kt = 0; kt < KT; ++kt, ++kk) {
                    const int st = kk % PS;
                    if (kk >= PS && !mbar_wait(&empty[st], ((kk / PS) & 1) ^ 1)) {
                        fail();
                        break;
                    }
                    const uint32_t sa = base + st * T::kStageBytes;
                    mbar_arrive_expect_tx(&full[st], tx);
                    tma_load_2d(sa, &tm_x, kt * KS, m0, &full[st]);
                    if (has_lo) tma_load_2d(sa + T::kXBytes, &tm_xlo, kt * KS, m0, &full[st]);
                    tma_load_2d_hint(sa + T::kWOffset, &tm_w, kt * KS, n0, &full[st], pol_w);
                    if (WLO) tma_load_2d_hint(sa + T::kWOffset + T::kWBytes, &tm_wlo, kt * KS, n0, &full[st], pol_w);
                    s_issued = kk + 1;
                }
            }
            grid_dep_launch();
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // ---- MMA issuer --------------------------------------------------------------------
            // M = 128 rows (A: activations), N = 256 features (B: weights), both K-major.
            const uint32_t idesc = p.a_f16 ? idesc_f16<NT2>() : idesc_bf16<NT2>();
            int kk = 0, i = 0;
            for (int t = blockIdx.x; t < tiles && !aborted(); t += gridDim.x, ++i) {
                const int acc = i & 1, use = i >> 1;
                if (use > 0 && !mbar_wait(&acc_empty[acc], (use - 1) & 1)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * NT2);
                bool ok = true;
                for (int kt = 0; kt < KT; ++kt, ++kk) {
                    const int st = kk % PS;
                    if (!mbar_wait(&full[st], (kk / PS) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = base + st * T::kStageBytes;
                    const uint64_t dx = sw128_desc(sa), dxl = sw128_desc(sa + T::kXBytes);
                    const uint64_t dw = sw128_desc(sa + T::kWOffset), dwl = sw128_desc(sa + T::kWOffset + T::kWBytes);
#pragma unroll
                    for (int k2 = 0; k2 < KS / 16; ++k2) {
                        tc_mma(d, dx + 2 * k2, dw + 2 * k2, idesc, (kt | k2) ? 1u : 0u);
                        if (has_lo) tc_mma(d, dxl + 2 * k2, dw + 2 * k2, idesc, 1u);
                        if (WLO) tc_mma(d, dx + 2 * k2, dwl + 2 * k2, idesc, 1u);
                    }
                    tc_commit(&empty[st]);
                    s_consumed = kk + 1;
                }
                if (!ok) {
                    fail();
                    break;
                }
                tc_commit(&acc_full[acc]);
            }
        }
    } else {
        // ---- epilogue ------------------------------------------------------------------------
        grid_dep_wait();  // the residual epilogues read what predecessors wrote
        const int ew = warp - 2, quarter = warp & 3, part = ew >> 2;
        float* stg = reinterpret_cast<float*>(smem + T::kStageOffset);
        int i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
            const int acc = i & 1, use = i >> 1;
            const int n0 = (t % NT) * NT2, m0 = (t / NT) * PT;
            const bool got = !aborted() && mbar_wait(&acc_full[acc], use & 1);
            if (!got) fail();
            if (epi_bar_any(!got)) break;  // every epilogue warp leaves together
            __syncwarp();
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < 8; ++c) {  // chunk c: rows 32 (c % 4) .., features 128 (c / 4) ..
                const int q = c & 3, h = c >> 2;
                if (quarter == q) {
                    float v[32];
                    tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * NT2 + 128 * h + 32 * part), v);
                    float4* row = reinterpret_cast<float4*>(stg + lane * kStageStride + 32 * part);
#pragma unroll
                    for (int j = 0; j < 8; ++j) row[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                }
                epi_bar_sync();
                if (EPI == EPI_QKV) qkv_rows(p, stg, n0 + 128 * h, m0 + 32 * q, ew);
                else plain_rows<EPI>(p, stg, n0 + 128 * h, m0 + 32 * q, 0, ew);
                epi_bar_sync();  // the chunk's readers are done with the staging tile
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        if (tid == 64) stamp_mark(p.stamps, p.stamp, STAMP_END);
    }

    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        // Copies issued but never consumed (only after a timeout): let them land before exit.
        for (int kk = s_consumed; kk < s_issued; ++kk) mbar_wait(&full[kk % PS], (kk / PS) & 1);
    }
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * NT2) : "memory");
    }
}

// ---- tensor maps ---------------------------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                 CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                 CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static const EncodeTiled fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<EncodeTiled>(f);
    }();
    return fn;
}

// Tensor map of a row-major [rows][cols] f16 (or bf16) matrix, box 64 (k) x box_rows, 128-byte
// swizzle, zero fill past the last row. A map is a pure function of its key, so cached maps never
// go stale; the cache is cleared when it grows large (prompt lengths vary).
bool f16_map(CUtensorMap* out, const void* ptr, int rows, int cols, int box_rows, bool bf16 = false) {
    using Key = std::tuple<const void*, int, int, int, bool>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{ptr, rows, cols, box_rows, bf16};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    EncodeTiled enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)KS, (cuuint32_t)box_rows};
    const cuuint32_t elem[2] = {1, 1};
    CUtensorMap m;
    if (enc(&m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
            const_cast<void*>(ptr), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return true;
}

// Tensor map of the row-major [rows][cols] int8 weights, box 64 (k, bytes) x box_rows, no
// swizzle: the box lands as box_rows dense rows of 64 bytes, which widen_w8 reads.
bool i8_map(CUtensorMap* out, const void* ptr, int rows, int cols, int box_rows, bool swizzle64 = false) {
    using Key = std::tuple<const void*, int, int, int, bool>;
    static std::mutex mu;
    static std::map<Key, CUtensorMap> cache;
    const Key key{ptr, rows, cols, box_rows, swizzle64};
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return true;
    }
    EncodeTiled enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols};
    const cuuint32_t box[2] = {(cuuint32_t)KS, (cuuint32_t)box_rows};
    const cuuint32_t elem[2] = {1, 1};
    CUtensorMap m;
    if (enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, elem,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return true;
}

// The weight map(s) of a launch: the int8 weights (kW8) or the 16-bit plane(s).
template <int WM>
bool weight_maps(const LinearArgs& a, CUtensorMap* mw, CUtensorMap* mwl) {
    if (WM == kW8) {
        if (!i8_map(mw, a.w, a.N, a.K, FT)) return false;
        *mwl = *mw;
        return true;
    }
    const bool bf = !a.a_f16;
    if (!f16_map(mw, a.wh, a.N, a.K, FT, bf)) return false;
    if (WM == kW16Lo) return f16_map(mwl, a.wh_lo, a.N, a.K, FT, bf);
    *mwl = *mw;
    return true;
}

template <int EPI, int RT, int WM>
bool launch_tma(const LinearArgs& a, cudaStream_t s) {
    using T = TmaTile<RT, WM>;
    const bool bf = !a.a_f16;
    CUtensorMap mw, mwl, mx, mxl;
    if (!weight_maps<WM>(a, &mw, &mwl) || !f16_map(&mx, a.a, a.M, a.K, RT, bf)) return false;
    if (a.a_lo) {
        if (!f16_map(&mxl, a.a_lo, a.M, a.K, RT, bf)) return false;
    } else {
        mxl = mx;
    }
    set_max_dynamic_smem(reinterpret_cast<const void*>(linear_tma_kernel<EPI, RT, WM>), T::kSmem);
    dim3 grid(a.N / FT, (a.M + RT - 1) / RT, a.splits);
    launch_k(linear_tma_kernel<EPI, RT, WM>, grid, dim3(kThreadsTma), T::kSmem, s, a, mw, mwl, mx, mxl);
    return true;
}

template <int EPI, int RT, bool Q8 = false>
bool launch_i8(const LinearArgs& a, cudaStream_t s) {
    using T = I8Tile<RT>;
    const bool bf = !a.a_f16;
    CUtensorMap mw, mx, mxl;
    if (!i8_map(&mw, a.w, a.N, a.K, FT, true) || !f16_map(&mx, a.a, a.M, a.K, RT, bf)) return false;
    mxl = mx;
    if (a.a_lo && !f16_map(&mxl, a.a_lo, a.M, a.K, RT, bf)) return false;
    set_max_dynamic_smem(reinterpret_cast<const void*>(linear_i8_kernel<EPI, RT, Q8>), T::kSmem);
    dim3 grid(a.N / FT, (a.M + RT - 1) / RT, a.splits);
    launch_k(linear_i8_kernel<EPI, RT, Q8>, grid, dim3(kThreadsTma), T::kSmem, s, a, mw, mx, mxl);
    return true;
}

// Prompt sizes: the persistent kernel, one CTA per SM over all tiles.
template <int EPI, int WM>
bool launch_persist(const LinearArgs& a, cudaStream_t s) {
    using T = PersistTile<WM>;
    const bool bf = !a.a_f16;
    CUtensorMap mw, mwl, mx, mxl;
    if (!weight_maps<WM>(a, &mw, &mwl) || !f16_map(&mx, a.a, a.M, a.K, PT, bf)) return false;
    mxl = mx;
    if (a.a_lo && !f16_map(&mxl, a.a_lo, a.M, a.K, PT, bf)) return false;
    set_max_dynamic_smem(reinterpret_cast<const void*>(linear_persist_kernel<EPI, WM>), T::kSmem);
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 1;
    const int tiles = (a.N / FT) * ((a.M + PT - 1) / PT);
    launch_k(linear_persist_kernel<EPI, WM>, dim3(tiles < sms ? tiles : sms), dim3(T::kThreads), T::kSmem, s, a,
             mw, mwl, mx, mxl);
    return true;
}

// Prompt sizes with 16-bit weights and N a multiple of 256: linear_rows_kernel.
template <int EPI, int WM>
bool launch_rows(const LinearArgs& a, cudaStream_t s) {
    using T = RowsTile<WM>;
    const bool bf = !a.a_f16;
    CUtensorMap mw, mwl, mx, mxl;
    if (!f16_map(&mw, a.wh, a.N, a.K, NT2, bf) || !f16_map(&mx, a.a, a.M, a.K, PT, bf)) return false;
    mwl = mw;
    if (WM == kW16Lo && !f16_map(&mwl, a.wh_lo, a.N, a.K, NT2, bf)) return false;
    mxl = mx;
    if (a.a_lo && !f16_map(&mxl, a.a_lo, a.M, a.K, PT, bf)) return false;
    set_max_dynamic_smem(reinterpret_cast<const void*>(linear_rows_kernel<EPI, WM>), T::kSmem);
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) sms = 1;
    const int tiles = (a.N / NT2) * ((a.M + PT - 1) / PT);
    launch_k(linear_rows_kernel<EPI, WM>, dim3(tiles < sms ? tiles : sms), dim3(T::kThreads), T::kSmem, s, a, mw,
             mwl, mx, mxl);
    return true;
}

// Whether prompt-size linears with 16-bit weights and N a multiple of 256 take linear_rows_kernel
// (default) or linear_persist_kernel (PTTS_B200_PERSIST=features).
bool rows_tiles() {
    static const bool on = [] {
        const char* e = getenv("PTTS_B200_PERSIST");
        return !(e && e[0] == 'f');
    }();
    return on;
}

// The weight form of a launch: 16-bit planes when the layer has them, else its int8 weights.
int weight_form(const LinearArgs& a) { return a.wh_lo ? kW16Lo : (a.wh ? kW16 : kW8); }

template <int EPI>
bool launch_tma_rows(const LinearArgs& a, cudaStream_t s) {
    // q8_0 values with block scales: only linear_i8_kernel's q8 form reads them (decode sizes).
    if (a.wblk) return a.a_f16 && a.M < kPersistMinRows && launch_i8<EPI, 32, true>(a, s);
    const int wm = weight_form(a);
    if (a.M >= kPersistMinRows && a.splits == 1 && EPI != EPI_PARTIAL) {
        if (wm != kW8 && a.N % NT2 == 0 && rows_tiles())
            return wm == kW16Lo ? launch_rows<EPI, kW16Lo>(a, s) : launch_rows<EPI, kW16>(a, s);
        if (wm == kW16Lo) return launch_persist<EPI, kW16Lo>(a, s);
        return wm == kW16 ? launch_persist<EPI, kW16>(a, s) : launch_persist<EPI, kW8>(a, s);
    }
    if (wm == kW16Lo) return launch_tma<EPI, 32, kW16Lo>(a, s);
    if (wm == kW16) return launch_tma<EPI, 32, kW16>(a, s);
    // int8 weights at decode sizes: widened into TMEM (linear_i8_kernel), or with
    // PTTS_B200_I8=smem in place in shared memory (linear_tma_kernel's kW8 form).
    const char* e = getenv("PTTS_B200_I8");
    return e && e[0] == 's' ? launch_tma<EPI, 32, kW8>(a, s) : launch_i8<EPI, 32>(a, s);
}

// The flow net's linears (bf16 planes, optional weight lo plane), decode-size rows only.
template <int EPI>
bool launch_tma_flow(const LinearArgs& a, cudaStream_t s) {
    return a.wh_lo ? launch_tma<EPI, 32, kW16Lo>(a, s) : launch_tma<EPI, 32, kW16>(a, s);
}

}  // namespace

bool bf16_rows_map(CUtensorMap* out, const void* ptr, long long rows, int cols, int box_cols, int box_rows,
                   int ld) {
    EncodeTiled enc = encoder();
    if (ld == 0) ld = cols;
    if (!enc || rows <= 0 || cols % 8 != 0 || ld % 8 != 0 || ld < cols || box_cols * 2 != 128) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return enc(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool linear_tc_supported(const LinearArgs& a) {
    return (a.wh != nullptr || a.w != nullptr) && a.M > 0 && a.N % FT == 0 && a.K % 8 == 0 && a.splits >= 1 &&
           a.K % a.splits == 0 && (a.K / a.splits) % KS == 0;
}

bool launch_linear_tc(const LinearArgs& a, LinearEpi epi, cudaStream_t s) {
    if (!linear_tc_supported(a)) return false;
    const bool flow_epi = epi >= EPI_BIAS;
    // A 16-bit weight plane has the activations' type: the layer stack's f16 copies pair only
    // with f16 planes. int8 weights are widened to whichever type the activations have.
    if (!flow_epi && !a.a_f16 && a.wh) return false;
    if (flow_epi && !a.wh) return false;  // the flow net's weights come as 16-bit planes
    switch (epi) {
        case EPI_F32: return launch_tma_rows<EPI_F32>(a, s);
        case EPI_QKV: return launch_tma_rows<EPI_QKV>(a, s);
        case EPI_RESID: return launch_tma_rows<EPI_RESID>(a, s);
        case EPI_GELU: return launch_tma_rows<EPI_GELU>(a, s);
        case EPI_PARTIAL: return launch_tma_rows<EPI_PARTIAL>(a, s);
        case EPI_BIAS: return launch_tma_flow<EPI_BIAS>(a, s);
        case EPI_COND: return launch_tma_flow<EPI_COND>(a, s);
        case EPI_BIAS_SILU: return launch_tma_flow<EPI_BIAS_SILU>(a, s);
        case EPI_GATE_RESID: return launch_tma_flow<EPI_GATE_RESID>(a, s);
    }
    return false;
}

}  // namespace ptts
