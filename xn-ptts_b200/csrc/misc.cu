// Row plans, length bookkeeping and small conversions.
#include <cstdlib>
#include <mutex>
#include <set>
#include <utility>

#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

constexpr int kPlanThreads = 1024;

// Open-addressing table of the repeated-stream check: keys, then the lowest row per key (dynamic
// shared memory, only in launches that ask for the check).
constexpr int kDupSlots = 2 * kPlanThreads;
constexpr int kDupSmemBytes = 2 * kDupSlots * (int)sizeof(int);

// One CTA: a running block scan over the sequences, 1024 at a time.
__global__ void __launch_bounds__(kPlanThreads) plan_decode_kernel(
    const int32_t* __restrict__ lengths, const int32_t* __restrict__ streams, int n,
    int num_streams, int capacity, RowPlan plan, RingArgs ring, int grid, uint32_t* err,
    PlanChecks chk) {
    __shared__ int warp_tot[kPlanThreads / 32];
    __shared__ int carry;
    extern __shared__ int dup_key[];
    int* dup_first = dup_key + kDupSlots;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    grid_dep_wait();
    grid_dep_launch();
    if (tid == 0) {
        carry = 0;
        plan.prefix[0] = 0;
    }
    // Repeated streams (n <= kPlanThreads): every row's stream goes into an open-addressing
    // table that keeps the lowest row index per stream; a row whose index is not the lowest
    // repeats an earlier row's stream. Probing ends within kDupSlots steps (at most n < kDupSlots
    // keys are ever inserted, so a free slot or the row's own key is always found).
    const bool unique = chk.unique && n <= kPlanThreads;
    int dup_slot = -1;
    if (unique) {
        for (int t = tid; t < kDupSlots; t += kPlanThreads) {
            dup_key[t] = -1;
            dup_first[t] = 0x7fffffff;
        }
        __syncthreads();
        if (tid < n) {
            const int sid = streams[tid];
            if (sid >= 0 && sid < num_streams) {
                int h = (int)(((unsigned)sid * 2654435761u) % (unsigned)kDupSlots);
                for (int t = 0; t < kDupSlots; ++t) {
                    const int prev = atomicCAS(&dup_key[h], -1, sid);
                    if (prev == -1 || prev == sid) {
                        atomicMin(&dup_first[h], tid);
                        dup_slot = h;
                        break;
                    }
                    h = h + 1 == kDupSlots ? 0 : h + 1;
                }
            }
        }
    }
    __syncthreads();
    for (int base = 0; base < n; base += kPlanThreads) {
        const int i = base + tid;
        int keys = 0;
        if (i < n) {
            const int sid = streams[i];
            bool refused = false;
            if (sid < 0 || sid >= num_streams) {
                set_error(err, DEV_ERR_BOUNDS);
                refused = true;
            } else if (unique && dup_slot >= 0 && dup_first[dup_slot] != i) {
                set_error(err, DEV_ERR_DUPLICATE);
                refused = true;
            }
            int len = 0, slot = 0;
            if (!refused) {
                len = lengths[sid];
                slot = len;
                keys = len + 1;
                const int w = ring.write ? ring.write[sid] : -1;
                const int ctx = ring.window ? ring.window[sid] : 0;
                if (len < 0) {
                    refused = true;
                } else if (w >= 0) {
                    if (w >= capacity) refused = true;
                    slot = w;
                    keys = min(max(ring.filled[sid], slot + 1), capacity);
                } else if (ctx > 0) {  // the position grows past the capacity; slots wrap
                    slot = len % capacity;
                    keys = min(min(len + 1, ctx), capacity);
                } else if (len + 1 > capacity) {
                    refused = true;
                }
                if (refused) set_error(err, DEV_ERR_CAPACITY);
            }
            if (refused) {
                keys = 0;
                plan.row_stream[i] = 0;
                plan.row_pos[i] = -1;
                plan.row_slot[i] = -1;
                if (chk.zero_out) {  // 4-byte stores: the decode kernel's own output alignment
                    uint32_t* o = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(chk.zero_out) +
                                                              (long long)i * chk.zero_row_bytes);
                    for (int t = 0; t < chk.zero_row_bytes / 4; ++t) o[t] = 0u;
                }
            } else {
                plan.row_stream[i] = sid;
                plan.row_pos[i] = len;
                plan.row_slot[i] = slot;
            }
        }
        int v = keys;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, v, o);
            if (lane >= o) v += t;
        }
        if (lane == 31) warp_tot[warp] = v;
        __syncthreads();
        if (warp == 0) {
            int w = warp_tot[lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o) w += t;
            }
            warp_tot[lane] = w;  // inclusive
        }
        __syncthreads();
        const int before = carry + (warp > 0 ? warp_tot[warp - 1] : 0);
        if (i < n) plan.prefix[i + 1] = before + v;
        __syncthreads();
        if (tid == 0) carry += warp_tot[kPlanThreads / 32 - 1];
        __syncthreads();
    }
    if (!plan.cta_first) return;
    // The CTAs of the decode launch: each starts in the stream holding its first key.
    const long long total = plan.prefix[n];
    const int G = ctas_in_use(total, grid);
    for (int b = tid; b < n; b += kPlanThreads) {
        const long long pb = plan.prefix[b], pe = plan.prefix[b + 1];
        if (pe <= pb) continue;
        for (int c = cta_of(pb, total, G); c <= cta_of(pe - 1, total, G); ++c)
            if (cta_start(c, total, G) >= pb) plan.cta_first[c] = b;
    }
}

__global__ void plan_rows_kernel(const int32_t* __restrict__ lengths,
                                 const int32_t* __restrict__ seq_stream,
                                 const int32_t* __restrict__ row_offsets, int n_seq, int n_rows,
                                 int num_streams, int capacity, RowPlan plan, const int32_t* window,
                                 uint32_t* err) {
    grid_dep_wait();
    grid_dep_launch();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n_rows) return;
    int lo = 0, hi = n_seq - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (row_offsets[mid] <= r) lo = mid;
        else hi = mid - 1;
    }
    int sid = seq_stream[lo];
    if (sid < 0 || sid >= num_streams) {
        set_error(err, DEV_ERR_BOUNDS);
        sid = 0;
    }
    const int pos = lengths[sid] + (r - row_offsets[lo]);
    const bool windowed = window && window[sid] > 0;
    if (pos < 0 || (!windowed && pos >= capacity)) set_error(err, DEV_ERR_CAPACITY);
    plan.row_stream[r] = sid;
    plan.row_pos[r] = pos;
    plan.row_slot[r] = windowed ? max(pos, 0) % capacity : pos;
}

__global__ void advance_kernel(int32_t* lengths, const int32_t* __restrict__ seq_stream,
                               const int32_t* __restrict__ row_offsets, int n_seq, int rows,
                               RingArgs ring, int capacity) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n_seq) return;
    const int add = row_offsets ? row_offsets[i + 1] - row_offsets[i] : rows;
    const int sid = seq_stream[i];
    const int w = ring.write ? ring.write[sid] : -1;
    if (w >= 0 && w < capacity) {
        ring.valid[(long long)sid * capacity + w] = 1;
        ring.filled[sid] = max(ring.filled[sid], w + 1);
    }
    lengths[sid] += add;
}

__global__ void ring_hide_kernel(RingEvictArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < a.n) a.ring.valid[(long long)a.sid * a.capacity + a.slots[i]] = 0;
    if (i == 0) a.lengths[a.sid] -= a.n;
}

// One thread per (layer, slot, pair); rotation arithmetic as the RoPE epilogues (rope.rs order).
template <typename T>
__global__ void ring_rotate_kernel(RingEvictArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const int pairs = a.row_elems / 2, slots = a.filled - a.prefix;
    const long long total = (long long)a.layers * slots * pairs;
    const uint8_t* valid = a.ring.valid + (long long)a.sid * a.capacity;
    T* k = static_cast<T*>(a.k_cache);
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int pr = (int)(i % pairs);
        const long long ls = i / pairs;
        const int slot = a.prefix + (int)(ls % slots), layer = (int)(ls / slots);
        if (!valid[slot]) continue;
        const int d2 = pr % (kHeadDim / 2);  // pair index within the head
        float sn, cs;
        sincosf((float)(-a.shift) * a.inv_freq[d2], &sn, &cs);
        T* e = k + layer * a.layer_elems + kv_offset(a.sid, slot, pr / (kHeadDim / 2), a.streams, a.capacity) +
               2 * d2;
        const float x0 = (float)e[0], x1 = (float)e[1];
        const float y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        const float y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        e[0] = (T)y0;
        e[1] = (T)y1;
    }
}

__global__ void set_lengths_kernel(int32_t* lengths, const int32_t* __restrict__ streams,
                                   const int32_t* __restrict__ values, int n) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) lengths[streams[i]] = values[i];
}

// The same for a short list passed in the kernel's parameters (no host-to-device copy).
__global__ void set_lengths_inline_kernel(int32_t* lengths, SetLengthsInline l) {
    grid_dep_wait();
    grid_dep_launch();
    const int i = threadIdx.x;
    if (i < l.n) lengths[l.stream[i]] = l.value[i];
}

__global__ void reset_streams_kernel(uint4* k, uint4* v, int32_t* lengths,
                                     const int32_t* __restrict__ streams, int n, int layers,
                                     long long layer_vec, long long stream_vec) {
    grid_dep_wait();
    grid_dep_launch();
    const long long per = stream_vec * layers;
    const long long total = per * n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int si = (int)(i / per);
        const long long rem = i - si * per;
        const int layer = (int)(rem / stream_vec);
        const long long off = layer * layer_vec + (long long)streams[si] * stream_vec +
                              (rem - layer * stream_vec);
        k[off] = make_uint4(0, 0, 0, 0);
        v[off] = make_uint4(0, 0, 0, 0);
        if (rem == 0) lengths[streams[si]] = 0;
    }
}

__global__ void bf16_to_f32_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ y,
                                   long long n) {
    grid_dep_wait();
    grid_dep_launch();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        y[i] = __bfloat162float(x[i]);
}

}  // namespace

void launch_plan_decode(const int32_t* lengths, const int32_t* streams, int n, int num_streams,
                        int capacity, RowPlan plan, const RingArgs& ring, int grid, uint32_t* err,
                        cudaStream_t s, const PlanChecks& checks) {
    PlanChecks c = checks;
    c.unique = c.unique && n <= kPlanThreads;
    launch_k(plan_decode_kernel, dim3(1), dim3(kPlanThreads), c.unique ? kDupSmemBytes : 0, s, lengths,
             streams, n, num_streams, capacity, plan, ring, grid < kMaxDecodeGrid ? grid : kMaxDecodeGrid,
             err, c);
}

void launch_plan_rows(const int32_t* lengths, const int32_t* seq_stream, const int32_t* row_offsets,
                      int n_seq, int n_rows, int num_streams, int capacity, RowPlan plan,
                      const int32_t* window, uint32_t* err, cudaStream_t s) {
    launch_k(plan_rows_kernel, dim3((n_rows + 255) / 256), dim3(256), 0, s, lengths, seq_stream,
             row_offsets, n_seq, n_rows, num_streams, capacity, plan, window, err);
}

void launch_advance(int32_t* lengths, const int32_t* seq_stream, const int32_t* row_offsets,
                    int n_seq, int rows, const RingArgs& ring, int capacity, cudaStream_t s) {
    launch_k(advance_kernel, dim3((n_seq + 255) / 256), dim3(256), 0, s, lengths, seq_stream,
             row_offsets, n_seq, rows, ring, capacity);
}

void launch_ring_evict(const RingEvictArgs& a, cudaStream_t s) {
    launch_k(ring_hide_kernel, dim3((a.n + 255) / 256 > 0 ? (a.n + 255) / 256 : 1), dim3(256), 0, s, a);
    if (a.filled <= a.prefix) return;
    const long long total = (long long)a.layers * (a.filled - a.prefix) * (a.row_elems / 2);
    const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
    if (a.bf16) launch_k(ring_rotate_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, s, a);
    else launch_k(ring_rotate_kernel<float>, dim3(blocks), dim3(256), 0, s, a);
}

void launch_set_lengths(int32_t* lengths, const int32_t* streams, const int32_t* values, int n,
                        cudaStream_t s) {
    launch_k(set_lengths_kernel, dim3((n + 255) / 256), dim3(256), 0, s, lengths, streams, values, n);
}

void launch_set_lengths_inline(int32_t* lengths, const SetLengthsInline& l, cudaStream_t s) {
    launch_k(set_lengths_inline_kernel, dim3(1), dim3(kSetLengthsInline), 0, s, lengths, l);
}

void launch_reset_streams(void* k, void* v, int32_t* lengths, const int32_t* streams, int n,
                          int layers, long long layer_bytes, long long stream_bytes,
                          cudaStream_t s) {
    launch_k(reset_streams_kernel, dim3(1184), dim3(256), 0, s, static_cast<uint4*>(k),
             static_cast<uint4*>(v), lengths, streams, n, layers, layer_bytes / 16,
             stream_bytes / 16);
}

__global__ void rope_table_kernel(RopeFreqs f, float2* __restrict__ out, int rows) {
    const long long n = (long long)rows * kMaxPairs;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int pos = (int)(i / kMaxPairs), k = (int)(i % kMaxPairs);
        float sn, cs;
        sincosf((float)pos * f.inv_freq[k], &sn, &cs);
        out[i] = make_float2(cs, sn);
    }
}

void launch_rope_table(RopeFreqs f, float2* out, int rows, cudaStream_t s) {
    const long long blocks = ((long long)rows * kMaxPairs + 255) / 256;
    rope_table_kernel<<<(int)(blocks < 4096 ? blocks : 4096), 256, 0, s>>>(f, out, rows);
}

__global__ void i8_to_f16_kernel(const int8_t* __restrict__ x, __half* __restrict__ y, long long n) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        y[i] = __short2half_rn((short)x[i]);
}

void launch_i8_to_f16(const int8_t* x, __half* y, long long n, cudaStream_t s) {
    const long long blocks = (n + 255) / 256;
    i8_to_f16_kernel<<<(int)(blocks < 4096 ? blocks : 4096), 256, 0, s>>>(x, y, n);
}

// 16 int8 -> 16 f16 per thread and step (one 16-byte load, two 16-byte stores).
__global__ void widen_i8_kernel(I8Widen w) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (int m = 0; m < 4; ++m) {
        const long long chunks = w.n[m] / 16;
        const uint4* src = reinterpret_cast<const uint4*>(w.src[m]);
        uint4* dst = reinterpret_cast<uint4*>(w.dst[m]);
        for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < chunks; i += stride) {
            const uint4 q = src[i];
            uint4 a, b;
            i8x4_to_f16x4(q.x, a.x, a.y);
            i8x4_to_f16x4(q.y, a.z, a.w);
            i8x4_to_f16x4(q.z, b.x, b.y);
            i8x4_to_f16x4(q.w, b.z, b.w);
            dst[2 * i] = a;
            dst[2 * i + 1] = b;
        }
    }
}

void launch_widen_i8(const I8Widen& w, cudaStream_t s) {
    widen_i8_kernel<<<1184, 256, 0, s>>>(w);
}

void launch_bf16_to_f32(const __nv_bfloat16* x, float* y, long long n, cudaStream_t s) {
    const long long blocks = (n + 255) / 256;
    launch_k(bf16_to_f32_kernel, dim3((int)(blocks < 4096 ? blocks : 4096)), dim3(256), 0, s, x, y, n);
}

void prefer_max_shared(const void* kernel) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (done.insert({dev, kernel}).second)
        cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
}

void set_max_dynamic_smem(const void* kernel, int bytes) {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (done.count({dev, kernel})) return;
    // Recorded only once set, so a launch on this device never precedes the attribute.
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess)
        done.insert({dev, kernel});
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("PTTS_B200_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

}  // namespace ptts
