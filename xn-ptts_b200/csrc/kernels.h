// Internal launchers of the ptts_b200 kernels (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "ptts_b200.h"

namespace ptts {

// Bits of the device-side error word. Kernels set these and return instead of trapping.
enum : uint32_t {
    DEV_ERR_BOUNDS = 1u,    // an index or position fell outside its buffer
    DEV_ERR_CAPACITY = 2u,  // a stream's rows did not fit its capacity
    DEV_ERR_TIMEOUT = 4u,   // a bounded mbarrier wait gave up
    DEV_ERR_DUPLICATE = 8u, // a stream appeared twice among one decode call's rows
};
static_assert(DEV_ERR_BOUNDS == PTTS_B200_DEVERR_BOUNDS && DEV_ERR_CAPACITY == PTTS_B200_DEVERR_CAPACITY &&
                  DEV_ERR_TIMEOUT == PTTS_B200_DEVERR_TIMEOUT && DEV_ERR_DUPLICATE == PTTS_B200_DEVERR_DUPLICATE,
              "device error bits match the C header");


// Launch with programmatic stream serialisation (PTTS_B200_PDL=0 turns it off): the kernel may
// start while its predecessor in the stream finishes; every kernel calls grid_dep_wait()
// before it reads what a predecessor wrote.
bool pdl_enabled();
// Asks, once per kernel and device, for the largest shared-memory carveout. Kernels of the two
// lanes of a step share SMs, and an SM runs CTAs side by side only under one carveout.
void prefer_max_shared(const void* kernel);
// Raises a kernel's dynamic shared-memory limit to `bytes`, once per kernel and device. Safe when
// host threads drive different devices at once (one object per device, one thread each).
void set_max_dynamic_smem(const void* kernel, int bytes);
template <typename... KArgs, typename... Args>
inline cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                            cudaStream_t s, Args&&... args) {
    prefer_max_shared(reinterpret_cast<const void*>(kernel));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Words of a kernel-timeline slot (stamp_mark): first entry, first start past the wait on the
// predecessor, and the complements of the last end and of the last entry.
enum { STAMP_ENTRY = 0, STAMP_START = 1, STAMP_END = 2, STAMP_LAST_ENTRY = 3 };

constexpr int kHeadDim = 64;   // D: the only head size the kernels implement
constexpr int kRowWidth = 512; // one cache row of a group of 8 heads (kGroupHeads * D)
constexpr int kGroupHeads = kRowWidth / kHeadDim;  // heads per group: 8
// Heads come in groups of 8. A layer's cache holds each group as one [streams][capacity][8][64]
// block, groups one after another, so every kernel reads a group's key or value rows as the
// contiguous 1 KB (bf16) rows of an 8-head layer. Element offset of (stream, slot, head) there:
__host__ __device__ inline long long kv_offset(int sid, int slot, int head, int num_streams, int capacity) {
    return (((long long)(head / kGroupHeads) * num_streams + sid) * capacity + slot) * kRowWidth +
           (head % kGroupHeads) * kHeadDim;
}
constexpr int kMaxPairs = kHeadDim / 2;

// Per-call row plan on the device: which arena stream, position and cache slot each row has.
struct RowPlan {
    int32_t* row_stream = nullptr;  // [rows]
    int32_t* row_pos = nullptr;     // [rows] RoPE position
    int32_t* row_slot = nullptr;    // [rows] cache slot written (the position, except in a ring)
    int32_t* prefix = nullptr;      // [rows + 1] decode only: prefix sums of attended keys
    int32_t* cta_first = nullptr;   // [kMaxDecodeGrid] decode only: the stream each CTA starts in
};
constexpr int kMaxDecodeGrid = 256;  // >= SMs of the GPU; the decode kernel's CTAs

// Ring caches (StreamingTransformer::start_ring / set_ring_slot / evict, transformer.rs:840-929):
// per stream the slot the next row goes to (-1: not a ring), one past the highest slot written,
// and which slots hold a row attention may see. nullptr members: no stream is a ring.
struct RingArgs {
    int32_t* write = nullptr;   // [streams]
    int32_t* filled = nullptr;  // [streams]
    uint8_t* valid = nullptr;   // [streams][capacity]
    // Windowed streams (Mimi's KvCache, transformer.rs:257-317): [streams] context, 0 = none. A
    // windowed stream writes position p at slot p % capacity and attends positions
    // max(0, p - context + 1) .. p.
    int32_t* window = nullptr;
};

// ---- plans and bookkeeping (misc.cu) ---------------------------------------------------

// Decode plan: one row per sequence. row_pos[i] = lengths[streams[i]]; the row is written at
// slot row_pos[i] and attends keys 0..row_pos[i]; a ring stream writes at its write slot w and
// attends slots 0..max(filled, w + 1) - 1 (the invisible ones masked by the decode kernel); a
// windowed stream writes at row_pos[i] % capacity and attends its last min(pos + 1, context)
// positions. prefix[i+1] = sum of attended keys.
// With plan.cta_first set, also cta_first[c] = the stream in which CTA c of a `grid`-CTA decode
// launch starts (the split-KV partition of the prefix sums), so no CTA searches for it.
//
// A row is refused when its stream index is out of range (DEV_ERR_BOUNDS), when, with
// PlanChecks::unique, an earlier row of the call names the same stream (DEV_ERR_DUPLICATE), or
// when its position does not fit the stream's slots (DEV_ERR_CAPACITY). A refused row attends
// no keys and writes no cache row (row_stream 0, row_pos and row_slot -1: the RoPE/append
// kernels and the QKV epilogues skip it), and with PlanChecks::zero_out its output row is
// written as zeros (no other kernel writes it).
struct PlanChecks {
    int unique = 0;            // check rows for repeated streams (n <= 1024 only)
    void* zero_out = nullptr;  // [n] rows of zero_row_bytes (a multiple of 4), or nullptr
    int zero_row_bytes = 0;
};
void launch_plan_decode(const int32_t* lengths, const int32_t* streams, int n, int num_streams,
                        int capacity, RowPlan plan, const RingArgs& ring, int grid, uint32_t* err,
                        cudaStream_t s, const PlanChecks& checks = PlanChecks{});

// Ragged plan: sequence i (stream seq_stream[i]) owns rows row_offsets[i]..row_offsets[i+1];
// row r of it sits at lengths[stream] + (r - row_offsets[i]).
// A windowed stream's row r sits at slot pos % capacity (window: [streams] contexts or nullptr).
void launch_plan_rows(const int32_t* lengths, const int32_t* seq_stream, const int32_t* row_offsets,
                      int n_seq, int n_rows, int num_streams, int capacity, RowPlan plan,
                      const int32_t* window, uint32_t* err, cudaStream_t s);

// lengths[seq_stream[i]] += rows (row_offsets == nullptr) or row_offsets[i+1]-row_offsets[i];
// for a ring stream also valid[write] = 1 and filled = max(filled, write + 1).
void launch_advance(int32_t* lengths, const int32_t* seq_stream, const int32_t* row_offsets,
                    int n_seq, int rows, const RingArgs& ring, int capacity, cudaStream_t s);

// Ring eviction of stream `sid` (transformer.rs:873-928): slots[0..n) become invisible, every
// still-visible key in slots [prefix, filled) of every layer is rotated back by n positions
// (RotaryEmbedding::shift_back, rope.rs:26-35: the rotation by -n, angle f32(-n) * inv_freq[i]),
// and lengths[sid] -= n.
struct RingEvictArgs {
    void* k_cache;            // all layers
    int layers;
    long long layer_elems;    // elements per layer
    int streams;              // streams of the arena (head groups: see kv_offset)
    int row_elems;            // H * D
    int capacity, sid, prefix, filled, shift;
    bool bf16;
    float inv_freq[kMaxPairs];
    const int32_t* slots;     // [n] device
    int n;
    RingArgs ring;
    int32_t* lengths;
};
void launch_ring_evict(const RingEvictArgs& a, cudaStream_t s);

// lengths[streams[i]] = values[i].
// Up to kSetLengthsInline (stream, value) pairs carried in the launch's parameters.
constexpr int kSetLengthsInline = 128;
struct SetLengthsInline {
    int n;
    int32_t stream[kSetLengthsInline];
    int32_t value[kSetLengthsInline];
};
void launch_set_lengths_inline(int32_t* lengths, const SetLengthsInline& l, cudaStream_t s);
void launch_set_lengths(int32_t* lengths, const int32_t* streams, const int32_t* values, int n,
                        cudaStream_t s);

// Zero `n` bytes of every listed stream's slots in every layer and set their lengths to 0.
void launch_reset_streams(void* k, void* v, int32_t* lengths, const int32_t* streams, int n,
                          int layers, long long layer_bytes, long long stream_bytes,
                          cudaStream_t s);

// bf16 -> f32 copy (the residual stream's start).
void launch_bf16_to_f32(const __nv_bfloat16* x, float* y, long long n, cudaStream_t s);

// ---- RoPE + append (rope_append.cu) ---------------------------------------------------

struct RopeAppendArgs {
    const void* q;         // [rows][H][D] in_dtype
    const void* k;         // [rows][KVH][D]
    const void* v;
    float* q_out;          // [rows][H][D] f32, rotated
    // Instead of q_out, when set: the rotated q times q_scale as bf16 hi and lo planes
    // [rows][H][D] (hi = bf16(x), lo = bf16(x - hi)), the form the tcgen05 prefill attention
    // copies by TMA (q_scale = log2(e) / sqrt(D): its scores come out in the exp2 domain).
    __nv_bfloat16* q_hi = nullptr;
    __nv_bfloat16* q_lo = nullptr;
    float q_scale = 1.f;
    void* k_cache;         // layer base [S][cap][H][D]
    void* v_cache;
    const int32_t* row_stream;
    const int32_t* row_pos;
    const int32_t* row_slot;   // cache slot of each row
    int rows, heads, kv_heads, num_streams, capacity;
    float inv_freq[kMaxPairs];
    uint32_t* err;
};
void launch_rope_append(const RopeAppendArgs& a, bool in_bf16, bool cache_bf16, cudaStream_t s);

// ---- attention (attn_decode.cu, attn_prefill.cu) -----------------------------------------

struct DecodeArgs {
    unsigned long long* stamps = nullptr;  // kernel timeline slot (see stamp_mark), or none
    int stamp = -1;
    const void* k_cache;      // this launch's head group of the layer: [S][cap][8][D]
    const void* v_cache;
    long long stream_bytes;   // capacity * row bytes
    const int32_t* row_stream;  // [B] arena stream of each sequence
    const int32_t* prefix;      // [B + 1] prefix sums of attended keys
    const float* q;           // [B][ld] f32, rotated: this launch's 8 heads from q
    void* out;                // [B][ld]: f32, bf16, or the hi plane (see out_mode)
    void* out_lo;             // [B][ld] bf16 lo plane when out_mode == kOutHiLo
    int out_mode;
    int ld = kRowWidth;       // elements from one row of q and out to the next (H * D)
    float* part;              // [(B + grid) * H * kPartStride]
    int* counters;            // [B * H], zero between launches (the merging warp resets its entry)
    const int32_t* cta_first = nullptr;  // [grid] the stream each CTA starts in, or nullptr (search)
    int B;
    float qscale;             // 1/sqrt(D) * log2(e)
    uint32_t* err;
    // Ring streams: key slot s is visible iff valid[s] or s == write (RingSlots::decode_mask,
    // transformer.rs:39-53). ring_write nullptr: no ring in the arena.
    const int32_t* ring_write = nullptr;
    const uint8_t* ring_valid = nullptr;
    int capacity = 0;
    // Windowed streams: the attended keys are positions pos + 1 - n .. pos of the row, at slots
    // modulo capacity (n = the row's key count). window nullptr: none in the arena.
    const int32_t* window = nullptr;
    const int32_t* row_pos = nullptr;
    // The plan and every cache row but the ones this launch's predecessor appends were written
    // before that predecessor began (it is not the plan kernel): the kernel reads the plan and
    // copies those rows before it waits for the predecessor.
    bool prestart = false;
};
// Output forms of the attention kernels.
constexpr int kOutF32 = 0, kOutBf16 = 1, kOutHiLo = 2;  // hi/lo: f16(o) and f16(o - hi)
constexpr int kPartStride = 68;  // floats per (slot, head) partial: acc[64], m, l, pad
// Split-KV decode over the balanced partition of all attended keys; the streams that span more
// than one CTA are merged by the CTA that finishes them last. `grid` CTAs at most (one per SM).
// `compact`: the smaller shared-memory ring, which leaves room on each SM for a linear's CTA.
void launch_decode_attn(const DecodeArgs& a, bool cache_bf16, int grid, cudaStream_t s, bool compact = false);
size_t decode_part_floats(int B, int grid);
size_t decode_counter_ints(int B);

struct PrefillArgs {
    const void* k_cache;      // this launch's head group of the layer: [S][cap][8][D]
    const void* v_cache;
    long long stream_elems;   // capacity * 8 * D
    const int32_t* row_stream;
    const int32_t* row_pos;
    const int32_t* window = nullptr;  // [streams] context of windowed streams (0: none)
    const float* q;           // [rows][H][D] f32, rotated
    // The same q times qscale as bf16 hi/lo planes [rows][H*D] (RopeAppendArgs::q_hi), which
    // the prefill_fa kernel copies by TMA (it needs them).
    const __nv_bfloat16* q_hi = nullptr;
    const __nv_bfloat16* q_lo = nullptr;
    void* out;                // [rows][ld] (see out_mode); q, q_hi, q_lo, out, out_lo start at
    void* out_lo;             // this launch's 8 heads
    int out_mode;
    int ld = kRowWidth;       // elements from one row of q (q_hi, q_lo) and out to the next
    int rows;
    float qscale;
    uint32_t* err;
};
// Causal attention of every row over keys 0..=row_pos, or over the last `context` positions
// (slots pos % capacity) for windowed streams (CUDA cores, online softmax).
void launch_prefill_attn(const PrefillArgs& a, bool cache_bf16, cudaStream_t s);
// The same on tcgen05 tiles, bf16 caches: one CTA per (tile of up to 128 consecutive rows of
// one sequence, head); tiles[i] = (first row, rows).
void launch_prefill_attn_tc(const PrefillArgs& a, const int2* tiles, int n_tiles, cudaStream_t s);
// The same with one CTA per (tile, group of heads), the group's (head, key tile) items in one
// pipeline (attn_prefill_fa.cu). `streams` and `capacity` describe the head group's cache block:
// [streams][capacity] rows of 512 bf16. False when the tensor maps cannot be made (nothing
// launched).
bool launch_prefill_attn_fa(const PrefillArgs& a, const int2* tiles, int n_tiles, int streams, int capacity,
                            cudaStream_t s);
// Tensor map of a row-major [rows][cols] bf16 matrix, box box_cols (128 bytes) x box_rows,
// 128-byte swizzle (linear_tc.cu).
bool bf16_rows_map(CUtensorMap* out, const void* ptr, long long rows, int cols, int box_cols, int box_rows,
                   int ld = 0);

// ---- int8 linear (linear.cu) ----------------------------------------------------------

enum LinearEpi : int {
    EPI_F32 = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_GELU = 3, EPI_PARTIAL = 4,
    // Flow net (bf16 planes, tcgen05 kernel only): y = W x + b; bf16 hi/lo of silu(W x + b + aux[n]);
    // bf16 hi/lo of silu(W x + b); y += aux[m * aux_stride + n] * (W x + b).
    EPI_BIAS = 5, EPI_COND = 6, EPI_BIAS_SILU = 7, EPI_GATE_RESID = 8
};

struct LinearArgs {
    unsigned long long* stamps = nullptr;  // kernel timeline slot (see stamp_mark), or none
    int stamp = -1;
    int M, N, K;
    int splits = 1;           // split-K slices (gridDim.z); EPI_PARTIAL writes slice z
    const void* a;            // A hi plane [M][K]: f16 (a_f16) or bf16
    const void* a_lo;         // A lo plane [M][K], or nullptr (A exact in one plane)
    int a_f16 = 1;            // 1: f16 planes (the layer stack); 0: one bf16 plane
    const int8_t* w;          // [N][K]
    const void* wh = nullptr;    // 16-bit weights [N][K] for the tcgen05 kernel (the f32 / q8_0 layers'
                                 // hi plane, the flow net's bf16 hi plane, or an f16 copy of w);
                                 // nullptr: the tcgen05 kernel widens the int8 `w` on chip
    const void* wh_lo = nullptr; // flow net: bf16 lo plane of the weights, or nullptr
    // q8_0 layers at decode sizes: `w` holds the q8_0 values and wblk [N][K / 32] each block's
    // scale divided by its row's power of two (`scale`), exact in f16; the tcgen05 kernel widens
    // q * d into the same f16 hi/lo weights as the layer's planes, on chip (a_f16 only).
    const __half* wblk = nullptr;
    const float* scale;       // [N], or nullptr (1) for the flow net
    const float* bias = nullptr;  // flow epilogues: [N] or nullptr
    const float* aux = nullptr;   // EPI_COND: time embedding [N]; EPI_GATE_RESID: gates
    int aux_stride = 0;           // EPI_GATE_RESID: row stride of aux
    float* y;                 // EPI_F32 / EPI_RESID: [M][N]; EPI_PARTIAL: [splits][M][N]
    void* yb;                 // EPI_GELU: f16 hi plane [M][N]
    void* yb_lo;              // EPI_GELU: f16 lo plane [M][N]
    float* yq;                // EPI_QKV: rotated q [M][H*D] f32
    __nv_bfloat16* yq_hi = nullptr;  // EPI_QKV: instead of yq, the rotated q times yq_scale as bf16
    __nv_bfloat16* yq_lo = nullptr;  //          hi/lo planes [M][H*D] (see RopeAppendArgs::q_hi)
    float yq_scale = 1.f;
    int gelu_tanh;
    // EPI_QKV
    const int32_t* row_stream;
    const int32_t* row_pos;
    const int32_t* row_slot;   // EPI_QKV: cache slot of each row
    __nv_bfloat16* k_cache;
    __nv_bfloat16* v_cache;
    int heads, kv_heads, num_streams, capacity;
    // (cos, sin)(f32(pos) * inv_freq[i]) at [pos][i] for pos < capacity (launch_rope_table):
    // the RoPE factors of the QKV epilogue, computed once per model instead of per element.
    const float2* rope;
    int rope_rows;  // positions in the table (>= capacity; more for windowed streams)
    uint32_t* err;
};
// N must be a multiple of 64 and K / splits a multiple of 64. launch_linear runs the TMA-fed
// tcgen05/TMEM kernel (linear_tc.cu) wherever linear_tc_supported holds (N a multiple of 128;
// int8 weights widened on chip, or 16-bit weight planes of the activations' type), and the
// mma.sync kernel (linear.cu) otherwise or when PTTS_B200_GEMM=mma. Layers loaded from f32 or
// q8_0 weights have no int8 copy (w == nullptr) and two f16 weight planes (wh, wh_lo): only the
// tcgen05 kernel takes them.
// From this many rows (one slice, not EPI_PARTIAL) the tcgen05 linears run the persistent
// kernel, which reads its weights only after the wait on its predecessor grid.
constexpr int kPersistMinRows = 4096;
bool launch_linear(const LinearArgs& a, LinearEpi epi, cudaStream_t s);  // false: nothing launched
void launch_linear_mma(const LinearArgs& a, LinearEpi epi, cudaStream_t s);
bool linear_tc_supported(const LinearArgs& a);
bool launch_linear_tc(const LinearArgs& a, LinearEpi epi, cudaStream_t s);  // false: not launched

// ---- flow head (flow.cu) ----------------------------------------------------------------
// y = a W^T + bias + add for K <= 64: a [M][K] (or every row a_row [K]), W [N][K] f32; output
// f32 y or bf16 yb.
struct FlowSmallArgs {
    int M, N, K;
    const float* a;
    const float* a_row;
    const float* w;
    const float* bias;
    const float* add;
    float* y;
    __nv_bfloat16* yb;
};
void launch_flow_small(const FlowSmallArgs& a, cudaStream_t s);

// Rows x [M][d] (LayerNorm with gamma/beta/eps first when gamma != nullptr) -> bf16 hi/lo planes
// and eos[m] = row . eos_w + eos_b. d in {128, 256, 512, 1024}.
struct FlowNormArgs {
    int M, d;
    const float* x;
    const float* gamma;
    const float* beta;
    float eps;
    const float* eos_w;
    float eos_b;
    float* eos;
    __nv_bfloat16* hi;
    __nv_bfloat16* lo;
};
void launch_flow_norm_eos(const FlowNormArgs& a, cudaStream_t s);

// LayerNorm(x) (eps; affine when gamma != nullptr) * (1 + scale) + shift, shift and scale rows
// at shift + m * stride, scale + m * stride; out f32 y, or bf16 hi/lo. C in {128, ..., 1024}.
struct FlowModArgs {
    int M, C;
    const float* x;
    const float* gamma;
    const float* beta;
    float eps;
    const float* shift;
    const float* scale;
    int stride;
    float* y;
    __nv_bfloat16* hi;
    __nv_bfloat16* lo;
};
void launch_flow_ln_mod(const FlowModArgs& a, cudaStream_t s);

// out[m][j] = cur[m][j] + step_scale * (h[m] . w[j] + bias[j]) (or the bare product when cur is
// nullptr); h [M][C], w [L][C], L <= 64, C * L * 4 <= 200 KB.
struct FlowOutArgs {
    int M, C, L;
    const float* h;
    const float* w;
    const float* bias;
    const float* cur;
    float step_scale;
    float* out;
};
void launch_flow_out(const FlowOutArgs& a, cudaStream_t s);
// The final layer's LayerNorm + modulate (`m`, no affine, no output: y, hi and lo unset) and the
// flow_out step (`o`, its h unused) in one kernel, for C = 512 and L <= 32; false (nothing
// launched) for other shapes.
bool launch_flow_final(const FlowModArgs& m, const FlowOutArgs& o, cudaStream_t s);

// RoPE table: out[pos][i] = (cos, sin)(f32(pos) * inv_freq[i]) for pos < rows, i < kMaxPairs.
struct RopeFreqs {
    float inv_freq[kMaxPairs];
};
void launch_rope_table(RopeFreqs f, float2* out, int rows, cudaStream_t s);

// int8 -> f16, exact (weights, once per layer load).
void launch_i8_to_f16(const int8_t* x, __half* y, long long n, cudaStream_t s);
// Up to four int8 matrices widened to f16 (exact) in one launch: n[i] a multiple of 16, src and
// dst 16-byte aligned. A plain launch (no programmatic serialisation): it starts after its
// predecessor in the stream has finished and its successor starts after it has.
struct I8Widen {
    const int8_t* src[4] = {};
    __half* dst[4] = {};
    long long n[4] = {};
};
void launch_widen_i8(const I8Widen& w, cudaStream_t s);

// Residual update and LayerNorm, one warp per row: resid = (x_bf16 ? x_bf16 : resid)
// + sum of `nsplit` partial slices [nsplit][M][d]; then, when hi != nullptr, LayerNorm(resid)
// (gamma, beta, eps 1e-5) written as f16 hi/lo planes. d in {128, 256, 512, 1024}.
struct LnArgs {
    unsigned long long* stamps = nullptr;  // kernel timeline slot (see stamp_mark), or none
    int stamp = -1;
    int M, d;
    float* resid;
    const __nv_bfloat16* x_bf16;
    const float* part;
    int nsplit;
    const float* gamma;
    const float* beta;
    __half* hi;
    __half* lo;
};
void launch_ln(const LnArgs& a, cudaStream_t s);

}  // namespace ptts
