// Split-KV decode attention: one query row per stream over that stream's cached keys
// 0..=pos, for a batch of streams with ragged lengths. A ring stream attends its slots
// 0..max(filled, write + 1) - 1 with the slots of evicted rows masked (RingSlots::decode_mask,
// transformer.rs:39-53). A windowed stream (Mimi's KvCache, transformer.rs:257-317) attends
// its last `context` positions, stored at slots modulo the capacity: a chunk that crosses the
// end of the slots is copied in two pieces.
//
// Reference: the t == 1 branch of StreamingMultiheadAttention::forward, `q.sdpa_decode(k, v,
// mask, 1/sqrt(d))` (ptts/src/transformer.rs:229-230), and its device-position twin at
// transformer.rs:216-224, which attends over every slot of the padded cache with a mask. Here
// only the filled keys are read: key j of a stream is visible iff j <= pos, which is what the
// mask of DeviceStep (transformer.rs:116-140) selects.
//
// Work split. All attended keys of the batch are laid end to end (prefix[b] .. prefix[b+1] for
// stream b) and cut into `G` equal ranges, one per CTA, so every CTA moves the same number of
// bytes whatever the length mix. A CTA walks the streams its range touches. A stream that lies
// wholly inside one range is finished there; the pieces of a stream cut by range ends leave
// partial (max, sum, acc) records at slot b + c (unique: along the key order each new piece
// increments b or c or both). The CTA that finishes a cut stream's last piece merges them: each
// piece's CTA publishes its records (threadfence) and bumps the stream's counter; the one that
// sees the count complete merges and resets the counter for the next launch. No CTA waits for
// another.
//
// Data movement. Keys and values of consecutive positions of a stream are contiguous
// (the cache is [stream][slot][head][dim]), so a chunk of positions is one 1-D bulk copy for K
// and one for V, issued by a producer warp into a shared-memory ring guarded by mbarriers (the
// wide or the compact ring, below). Eight consumer warps, one per head, read their head's
// 128-byte slice of every row with 16-byte shared loads (8 lanes per row, 4 rows per warp
// instruction) and keep an online softmax in the exp2 domain. Every wait is bounded and reports
// DEV_ERR_TIMEOUT.
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int kHeads = kRowWidth / kHeadDim;  // 8
constexpr int kConsumerWarps = kHeads;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kQStageBytes = kHeads * kHeadDim * 4;      // the f32 q of a stream a piece starts
constexpr int kHdrBytes = 128;                           // the chunk's header

// The shared-memory ring: STAGES stages of DATA bytes (K half + V half of a chunk) plus the q
// and header slots. The wide ring (3 x 64 KB) is for a kernel that has the SMs to itself; the
// compact one (4 x 32 KB, 137 KB) leaves room on every SM for a linear's CTA (74 KB) of a
// step's other lane, so the two run side by side. STAGED: consumers copy their slices of a
// chunk into registers and hand the stage back before scoring the rows, so the small ring
// stays nearly full of copies in flight (measured: +0.5 % on a two-lane frame; -2 % for the
// wide ring alone, which keeps scoring from shared memory).
template <int STAGES, int DATA, bool STAGED>
struct Ring {
    static constexpr int kStages = STAGES;
    static constexpr int kDataBytes = DATA;
    static constexpr bool kStaged = STAGED;
    static constexpr int kStageBytes = DATA + kQStageBytes + kHdrBytes;
    static constexpr int kSmemBytes = STAGES * kStageBytes + 2 * STAGES * 8;
    static_assert(kStageBytes % 128 == 0, "stages stay 128-byte aligned");
};
using WideRing = Ring<3, 64 * 1024, false>;
using CompactRing = Ring<4, 32 * 1024, true>;

// What the producer tells the consumers about a chunk (written before the stage's arrive, read
// after its wait): stream b of the batch, rows p .. p + n - 1 of its attended keys.
struct ChunkHdr {
    int b, p, n, flags;
    int sid;         // arena stream
    int ring_w;      // ring write slot, or -1
    int c0, c1;      // the CTAs holding pieces of a cut stream
};
constexpr int kFirst = 1, kLast = 2, kWhole = 4, kEnd = 8;
constexpr int kQLoaded = 16;  // the consumers loaded this piece's q themselves (none in the stage)

template <typename T>
struct Row;
template <>
struct Row<__nv_bfloat16> {
    static constexpr int kBytes = kRowWidth * 2;  // 1 KB
};
template <>
struct Row<float> {
    static constexpr int kBytes = kRowWidth * 4;  // 2 KB
};

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Eight elements of a head row for lane slice j, as stored (one 16-byte slice of bf16, two of
// f32), and widened: bf16 dims 8j..8j+7; f32 dims 4j..4j+3 and 32+4j..32+4j+3 (two 16-byte
// loads that stay conflict-free).
template <typename T>
struct Raw;
template <>
struct Raw<__nv_bfloat16> {
    uint4 u;
};
template <>
struct Raw<float> {
    float4 a, b;
};
__device__ __forceinline__ void load_raw(const unsigned char* head_row, int j, Raw<__nv_bfloat16>& r) {
    r.u = *reinterpret_cast<const uint4*>(head_row + 16 * j);
}
__device__ __forceinline__ void load_raw(const unsigned char* head_row, int j, Raw<float>& r) {
    r.a = *reinterpret_cast<const float4*>(head_row + 16 * j);
    r.b = *reinterpret_cast<const float4*>(head_row + 128 + 16 * j);
}
__device__ __forceinline__ void widen(const Raw<__nv_bfloat16>& r, float* o) {
    const uint4 u = r.u;
    o[0] = bf16lo(u.x); o[1] = bf16hi(u.x); o[2] = bf16lo(u.y); o[3] = bf16hi(u.y);
    o[4] = bf16lo(u.z); o[5] = bf16hi(u.z); o[6] = bf16lo(u.w); o[7] = bf16hi(u.w);
}
__device__ __forceinline__ void widen(const Raw<float>& r, float* o) {
    o[0] = r.a.x; o[1] = r.a.y; o[2] = r.a.z; o[3] = r.a.w;
    o[4] = r.b.x; o[5] = r.b.y; o[6] = r.b.z; o[7] = r.b.w;
}
// The f32 q slice that matches widen's dims for lane slice j.
template <typename T>
__device__ __forceinline__ void load_q(const float* qh, int j, float* o) {
    const float4 a = *reinterpret_cast<const float4*>(qh + (sizeof(T) == 2 ? 8 * j : 4 * j));
    const float4 b = *reinterpret_cast<const float4*>(qh + (sizeof(T) == 2 ? 8 * j + 4 : 32 + 4 * j));
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}

template <typename T>
__device__ __forceinline__ int dim_of(int j, int i) {
    if (sizeof(T) == 2) return 8 * j + i;
    return i < 4 ? 4 * j + i : 32 + 4 * j + (i - 4);
}

template <typename T>
__device__ __forceinline__ void store_out(const DecodeArgs& a, long long at, int j, const float* v) {
    if (a.out_mode == kOutF32) {
        float* o = static_cast<float*>(a.out) + at;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[dim_of<T>(j, i)] = v[i];
        return;
    }
    if (a.out_mode == kOutBf16) {
        __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + at;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[dim_of<T>(j, i)] = __float2bfloat16_rn(v[i]);
        return;
    }
    __half* o = static_cast<__half*>(a.out) + at;
    __half* ol = static_cast<__half*>(a.out_lo) + at;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float hf, lf;
        split_f16(v[i], hf, lf);
        o[dim_of<T>(j, i)] = __float2half_rn(hf);
        ol[dim_of<T>(j, i)] = __float2half_rn(lf);
    }
}

// Merge the partial records of stream b, head h, written by CTAs c0..c1 (one warp; lane owns
// dims 2*lane, 2*lane+1). Records of other CTAs are read past L1.
__device__ __forceinline__ void merge_head(const DecodeArgs& a, int b, int h, int c0, int c1, int lane) {
    float mx = -1e30f;
    for (int c = c0; c <= c1; ++c)
        mx = fmaxf(mx, __ldcg(a.part + ((long long)(b + c) * kHeads + h) * kPartStride + 64));
    float n0 = 0.f, n1 = 0.f, den = 0.f;
    for (int c = c0; c <= c1; ++c) {
        const float* rec = a.part + ((long long)(b + c) * kHeads + h) * kPartStride;
        const float f = fast_exp2(__ldcg(rec + 64) - mx);
        den += f * __ldcg(rec + 65);
        n0 += f * __ldcg(rec + 2 * lane);
        n1 += f * __ldcg(rec + 2 * lane + 1);
    }
    const float inv = 1.f / den;
    const long long at = (long long)b * a.ld + h * kHeadDim + 2 * lane;
    const float o0 = n0 * inv, o1 = n1 * inv;
    if (a.out_mode == kOutF32) {
        *reinterpret_cast<float2*>(static_cast<float*>(a.out) + at) = make_float2(o0, o1);
    } else if (a.out_mode == kOutBf16) {
        *reinterpret_cast<uint32_t*>(static_cast<__nv_bfloat16*>(a.out) + at) = pack_bf16x2(o0, o1);
    } else {
        uint32_t hi, lo;
        split_f16x2(o0, o1, hi, lo);
        *reinterpret_cast<uint32_t*>(static_cast<__half*>(a.out) + at) = hi;
        *reinterpret_cast<uint32_t*>(static_cast<__half*>(a.out_lo) + at) = lo;
    }
}

template <typename T, class R>
__global__ void __launch_bounds__(kThreads, 1) decode_attn_kernel(DecodeArgs a) {
    constexpr int kStages = R::kStages, kDataBytes = R::kDataBytes, kStageBytes = R::kStageBytes;
    constexpr int RB = Row<T>::kBytes;
    constexpr int HB = RB / kHeads;              // one head of one row: 128 or 256 bytes
    constexpr int CH = kDataBytes / 2 / RB;      // rows per chunk: wide 32 (bf16) or 16 (f32), compact 16 or 8
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
    uint64_t* empty = full + kStages;
    // With `prestart` the plan is complete before the predecessor began, so it is read now; the
    // producer waits for the predecessor (which writes q and this step's cache rows) only before
    // the first copy that needs either.
    if (threadIdx.x == 0) stamp_mark(a.stamps, a.stamp, STAMP_ENTRY);
    if (!a.prestart) grid_dep_wait();
    if (!a.prestart && threadIdx.x == 0) stamp_mark(a.stamps, a.stamp, STAMP_START);
    const long long total = a.prefix[a.B];
    const int G = ctas_in_use(total, gridDim.x);
    const int c = blockIdx.x;
    if (c >= G) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---- producer: one lane walks this CTA's key range and issues the bulk copies -------
        if (lane != 0) return;
        const long long start = cta_start(c, total, G), end = cta_start(c + 1, total, G);
        int b0 = a.cta_first ? a.cta_first[c] : 0;
        if (!a.cta_first) {  // the last stream whose keys begin at or before `start`
            int lo = 0, hi = a.B - 1;
            while (lo < hi) {
                const int mid = (lo + hi + 1) >> 1;
                if (a.prefix[mid] <= start) lo = mid;
                else hi = mid - 1;
            }
            b0 = lo;
        }
        const uint64_t pol = policy_evict_first();
        const unsigned char* kc = static_cast<const unsigned char*>(a.k_cache);
        const unsigned char* vc = static_cast<const unsigned char*>(a.v_cache);
        int it = 0;
        bool ok = true;
        auto stage_free = [&](int k) {  // wait until the consumers have released stage k % S
            if (mbar_wait(&empty[k % kStages], ((k / kStages) & 1) ^ 1)) return true;
            set_error(a.err, DEV_ERR_TIMEOUT);
            return false;
        };
        // Before the wait: the stages (at most kStages) whose q copy is still to be issued. The
        // consumers load the q of the CTA's first piece themselves as soon as they are past the
        // wait (plain loads, not queued behind the K/V copies), so that piece has none staged.
        const bool q_first_loaded = a.prestart && a.cta_first != nullptr;
        bool waited = !a.prestart;
        int q_stage[kStages], q_row[kStages], n_deferred = 0;
        auto wait_predecessor = [&]() {
            grid_dep_wait();
            stamp_mark(a.stamps, a.stamp, STAMP_START);
            waited = true;
            for (int i = 0; i < n_deferred; ++i)
                bulk_g2s(smem + q_stage[i] * kStageBytes + kDataBytes, a.q + (long long)q_row[i] * a.ld,
                         kQStageBytes, &full[q_stage[i]], pol);
        };
        for (int b = b0; b < a.B && ok; ++b) {
            const long long pb = a.prefix[b], pe = a.prefix[b + 1];
            if (pb >= end) break;
            const int s0 = (int)((start > pb ? start : pb) - pb);
            const int s1 = (int)((end < pe ? end : pe) - pb);
            const bool whole = pb >= start && pe <= end;
            const int sid = a.row_stream[b];
            const long long base = (long long)sid * a.stream_bytes;
            // Key i of the stream sits at slot i, or for a windowed stream at slot
            // (first + i) % capacity, first being the oldest attended position.
            const bool wrap = a.window && a.capacity > 0 && a.window[sid] > 0;
            const int first = wrap ? (int)(((long long)a.row_pos[b] + 1 - (pe - pb)) % a.capacity) : 0;
            ChunkHdr proto;
            proto.b = b;
            proto.sid = sid;
            proto.ring_w = a.ring_write ? a.ring_write[sid] : -1;
            proto.c0 = whole ? c : cta_of(pb, total, G);
            proto.c1 = whole ? c : cta_of(pe - 1, total, G);
            for (int p = s0; p < s1; p += CH, ++it) {
                const int n = min(CH, s1 - p);
                const int st = it % kStages;
                // The row this step appends: the ring's write slot, else the stream's last key.
                const bool new_row = proto.ring_w >= 0 ? (p <= proto.ring_w && proto.ring_w < p + n)
                                                       : p + n == (int)(pe - pb);
                if (!waited && (it >= kStages || new_row)) wait_predecessor();
                if (!(ok = stage_free(it))) break;
                unsigned char* sb = smem + st * kStageBytes;
                ChunkHdr hd = proto;
                hd.p = p;
                hd.n = n;
                const bool q_loaded = it == 0 && q_first_loaded;  // the CTA's first chunk: stream b0
                hd.flags = (p == s0 ? kFirst : 0) | (p + n >= s1 ? kLast : 0) | (whole ? kWhole : 0) |
                           (q_loaded ? kQLoaded : 0);
                *reinterpret_cast<ChunkHdr*>(sb + kDataBytes + kQStageBytes) = hd;
                mbar_arrive_expect_tx(&full[st], 2u * n * RB + (p == s0 && !q_loaded ? (uint32_t)kQStageBytes : 0u));
                if (p == s0 && !q_loaded) {
                    if (waited) {
                        bulk_g2s(sb + kDataBytes, a.q + (long long)b * a.ld, kQStageBytes, &full[st], pol);
                    } else {
                        q_stage[n_deferred] = st;
                        q_row[n_deferred++] = b;
                    }
                }
                const int slot = wrap ? (first + p) % a.capacity : p;
                const int n0 = wrap ? min(n, a.capacity - slot) : n;  // rows before the wrap
                bulk_g2s(sb, kc + base + (long long)slot * RB, n0 * RB, &full[st], pol);
                bulk_g2s(sb + kDataBytes / 2, vc + base + (long long)slot * RB, n0 * RB, &full[st], pol);
                if (n0 < n) {
                    bulk_g2s(sb + n0 * RB, kc + base, (n - n0) * RB, &full[st], pol);
                    bulk_g2s(sb + kDataBytes / 2 + n0 * RB, vc + base, (n - n0) * RB, &full[st], pol);
                }
            }
        }
        if (!waited) wait_predecessor();
        if (ok && stage_free(it)) {  // the end of the range: a header alone
            const int st = it % kStages;
            reinterpret_cast<ChunkHdr*>(smem + st * kStageBytes + kDataBytes + kQStageBytes)->flags = kEnd;
            mbar_arrive(&full[st]);
            ++it;
        }
        // Every copy is issued: the next kernel may launch (its CTAs wait for this grid).
        grid_dep_launch();
        // Before leaving, let every copy still in flight land (bounded) so none writes into
        // shared memory of a CTA that has gone.
        for (int k = (it > kStages ? it - kStages : 0); k < it; ++k)
            if (!mbar_wait(&full[k % kStages], (k / kStages) & 1)) set_error(a.err, DEV_ERR_TIMEOUT);
        return;
    }

    // ---- consumers: warp h owns head h and follows the producer's chunks --------------------
    // No CTA-wide barrier after the start: a warp whose wait times out leaves on its own.
    if (a.prestart) grid_dep_wait();
    const int h = warp;
    const int g = lane >> 3;  // which of the 4 rows of a warp step
    const int j = lane & 7;   // which 16-byte slice of the head row
    float q[8], m = -1e30f, l = 0.f, acc[8];
    // The q of the CTA's first piece (stream cta_first[c]), loaded now rather than staged.
    float q_first[8];
    if (a.prestart && a.cta_first) {
        const int b0 = min(max(a.cta_first[c], 0), max(a.B - 1, 0));
        load_q<T>(a.q + (long long)b0 * a.ld + h * kHeadDim, j, q_first);
    }
    for (int it = 0;; ++it) {
        const int st = it % kStages;
        if (!mbar_wait(&full[st], (it / kStages) & 1)) {
            set_error(a.err, DEV_ERR_TIMEOUT);
            break;
        }
        const unsigned char* sb = smem + st * kStageBytes;
        const ChunkHdr hd = *reinterpret_cast<const ChunkHdr*>(sb + kDataBytes + kQStageBytes);
        if (hd.flags & kEnd) break;
        if (hd.flags & kFirst) {
            if (hd.flags & kQLoaded) {
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = q_first[i];
            } else {
                load_q<T>(reinterpret_cast<const float*>(sb + kDataBytes) + h * kHeadDim, j, q);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] *= a.qscale;
            m = -1e30f;
            l = 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        }
        // Ring stream: slot s is visible iff valid[s] or s is the slot being written.
        const uint8_t* vis = hd.ring_w >= 0 ? a.ring_valid + (long long)hd.sid * a.capacity : nullptr;
        const int n = hd.n, p = hd.p;
        const unsigned char* ks = sb + h * HB;
        const unsigned char* vs = ks + kDataBytes / 2;
        // Row 4i + g of the chunk is lane group g's i-th row (rows past n repeat row n - 1 and
        // are masked). A staged ring's slices go to registers first and the stage goes back to
        // the producer at once: it refills the stage while these rows are scored.
        constexpr int RPL = CH / 4;
        static_assert(CH % 8 == 0, "rows are scored two per lane group at a time");
        Raw<T> kr[R::kStaged ? RPL : 1], vr[R::kStaged ? RPL : 1];
        if constexpr (R::kStaged) {
#pragma unroll
            for (int i = 0; i < RPL; ++i) {
                const int r = 4 * i + g;
                const int rr = r < n ? r : n - 1;
                load_raw(ks + rr * RB, j, kr[i]);
                load_raw(vs + rr * RB, j, vr[i]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
#pragma unroll
        for (int i = 0; i < RPL; i += 2) {
            if (4 * i >= n) break;
            const int r0 = 4 * i + g, r1 = 4 * i + 4 + g;
            const int rr0 = r0 < n ? r0 : n - 1, rr1 = r1 < n ? r1 : n - 1;
            Raw<T> rk0, rk1, rv0, rv1;
            if constexpr (R::kStaged) {
                rk0 = kr[i], rk1 = kr[i + 1], rv0 = vr[i], rv1 = vr[i + 1];
            } else {
                load_raw(ks + rr0 * RB, j, rk0);
                load_raw(ks + rr1 * RB, j, rk1);
            }
            float k0[8], k1[8];
            widen(rk0, k0);
            widen(rk1, k1);
            float d0 = 0.f, d1 = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                d0 = fmaf(q[e], k0[e], d0);
                d1 = fmaf(q[e], k1[e], d1);
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                d0 += __shfl_xor_sync(0xffffffffu, d0, o);
                d1 += __shfl_xor_sync(0xffffffffu, d1, o);
            }
            if (r0 >= n) d0 = -INFINITY;
            if (r1 >= n) d1 = -INFINITY;
            if (vis) {
                const int s0 = p + rr0, s1 = p + rr1;
                if (!vis[s0] && s0 != hd.ring_w) d0 = -INFINITY;
                if (!vis[s1] && s1 != hd.ring_w) d1 = -INFINITY;
            }
            const float mn = fmaxf(m, fmaxf(d0, d1));
            const float corr = fast_exp2(m - mn);
            const float e0 = fast_exp2(d0 - mn), e1 = fast_exp2(d1 - mn);
            l = fmaf(l, corr, e0 + e1);
            if constexpr (!R::kStaged) {
                load_raw(vs + rr0 * RB, j, rv0);
                load_raw(vs + rr1 * RB, j, rv1);
            }
            float v0[8], v1[8];
            widen(rv0, v0);
            widen(rv1, v1);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] = fmaf(e1, v1[e], fmaf(e0, v0[e], acc[e] * corr));
            m = mn;
        }
        if constexpr (!R::kStaged) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[st]);
        }
        if (!(hd.flags & kLast)) continue;
        // The end of this CTA's piece of stream b: merge the four row groups (lanes j, j+8,
        // j+16, j+24 hold the same dims).
        float mm = m, ll = l, aa[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) aa[i] = acc[i];
#pragma unroll
        for (int o = 8; o <= 16; o <<= 1) {
            const float mo = __shfl_xor_sync(0xffffffffu, mm, o);
            const float lo = __shfl_xor_sync(0xffffffffu, ll, o);
            const float mn = fmaxf(mm, mo);
            const float fa = fast_exp2(mm - mn), fb = fast_exp2(mo - mn);
            ll = ll * fa + lo * fb;
#pragma unroll
            for (int i = 0; i < 8; ++i) aa[i] = aa[i] * fa + __shfl_xor_sync(0xffffffffu, aa[i], o) * fb;
            mm = mn;
        }
        const int b = hd.b;
        if (hd.flags & kWhole) {
            if (g == 0) {
                const float inv = 1.f / ll;
#pragma unroll
                for (int i = 0; i < 8; ++i) aa[i] *= inv;
                store_out<T>(a, (long long)b * a.ld + h * kHeadDim, j, aa);
            }
            continue;
        }
        // A cut stream: publish this head's piece; the warp that completes the head's count
        // over the stream's pieces merges them and resets the count for the next launch.
        if (g == 0) {
            float* rec = a.part + ((long long)(b + c) * kHeads + h) * kPartStride;
#pragma unroll
            for (int i = 0; i < 8; ++i) rec[dim_of<T>(j, i)] = aa[i];
            if (j == 0) {
                rec[64] = mm;
                rec[65] = ll;
            }
        }
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            int* cnt = a.counters + (long long)b * kHeads + h;
            last = atomicAdd(cnt, 1) + 1 == hd.c1 - hd.c0 + 1;
            if (last) *cnt = 0;
        }
        if (__shfl_sync(0xffffffffu, last, 0)) {
            __threadfence();
            merge_head(a, b, h, hd.c0, hd.c1, lane);
        }
    }
    if (lane == 0) stamp_mark(a.stamps, a.stamp, STAMP_END);
}

template <typename T, class R>
void launch_typed(const DecodeArgs& a, int grid, cudaStream_t s) {
    set_max_dynamic_smem(reinterpret_cast<const void*>(decode_attn_kernel<T, R>), R::kSmemBytes);
    launch_k(decode_attn_kernel<T, R>, dim3(grid), dim3(kThreads), R::kSmemBytes, s, a);
}

}  // namespace

size_t decode_counter_ints(int B) { return (size_t)B * kHeads; }

size_t decode_part_floats(int B, int grid) {
    return (size_t)(B + grid) * kHeads * kPartStride;
}

void launch_decode_attn(const DecodeArgs& a, bool cache_bf16, int grid, cudaStream_t s, bool compact) {
    if (compact) {
        if (cache_bf16) launch_typed<__nv_bfloat16, CompactRing>(a, grid, s);
        else launch_typed<float, CompactRing>(a, grid, s);
    } else {
        if (cache_bf16) launch_typed<__nv_bfloat16, WideRing>(a, grid, s);
        else launch_typed<float, WideRing>(a, grid, s);
    }
}

}  // namespace ptts
