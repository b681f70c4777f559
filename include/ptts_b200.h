/*
 * ptts_b200 — B200 (sm_100a) kernels for the flow-LM attention path of Phonon TTS
 * (gradium-ai/xn-ptts), behind a plain C ABI.
 *
 * The reference composes this path from `xn` tensor ops inside
 *   ptts/src/transformer.rs:183-251  StreamingMultiheadAttention::forward
 *   ptts/src/transformer.rs:591-634  StreamingTransformerLayer::forward
 *   ptts/src/transformer.rs:742-838  StreamingTransformer::{forward, forward_step}
 * and keeps its KV cache in StreamingTransformerState (transformer.rs:12-25, 328-393).
 * This header replaces those with two objects and a handful of calls:
 *
 *   ptts_b200_kv     the per-layer K/V caches of many independent streams plus one
 *                    length per stream (StreamingMHAState::current_end), resident in HBM;
 *   ptts_b200_model  the flow-LM transformer's weights (int8, one f32 scale per output row).
 *
 * Conventions (mirroring ptts-ffi/include/ptts.h:28-52 and ptts-ffi/src/lib.rs:57-71):
 *   - every call returns an int status: PTTS_B200_OK (0) or a negative PTTS_B200_ERR_*;
 *   - on failure ptts_b200_last_error() returns a message for the calling thread;
 *   - no C++ exception crosses this boundary;
 *   - tensors passed as `const void*` / `void*` are DEVICE pointers unless the parameter name
 *     ends in `_host`; `cuda_stream` is a cudaStream_t (NULL = the legacy default stream);
 *   - calls on one object are serialised by the caller (one generation per session, as the
 *     reference's in-flight guard enforces at ptts/src/synth.rs:958-975).
 *
 * Layouts. K/V caches: [num_layers][num_heads / 8][num_streams][capacity][8][head_dim]: per
 * layer the layout of StreamingMHAState::k_cache ([num_streams][capacity][num_heads][head_dim],
 * transformer.rs:15-18) when num_heads is 8, and for more heads one such block per group of 8
 * heads (heads 8g .. 8g + 7 in block g), so that every position's row of a group is 1 KB (bf16)
 * of contiguous memory. Rows of q/k/v or hidden states are row-major with heads-major, then
 * head_dim, within a row (transformer.rs:197-211).
 *
 * Supported shapes: head_dim 64 and num_heads a multiple of 8 (8 in the 31m/40m flow LMs, 16 in
 * the reference's 1024-wide test config); d_model and dim_feedforward multiples of 64;
 * num_kv_heads dividing num_heads. Others are refused with PTTS_B200_ERR_UNSUPPORTED.
 */
#ifndef PTTS_B200_H
#define PTTS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PTTS_B200_OK 0
#define PTTS_B200_ERR_ARG (-1)         /* a bad argument: NULL, negative, out of range */
#define PTTS_B200_ERR_CAPACITY (-2)    /* rows do not fit a stream's capacity */
#define PTTS_B200_ERR_CUDA (-3)        /* a CUDA runtime call failed */
#define PTTS_B200_ERR_STATE (-4)       /* missing weights, mismatched objects, wrong order */
#define PTTS_B200_ERR_UNSUPPORTED (-5) /* a shape or type these kernels do not implement */
#define PTTS_B200_ERR_DEVICE (-6)      /* a kernel's own bounds check or bounded wait tripped */

/* Bits of the device-side error word (ptts_b200_kv_check reads the kv's own word;
 * ptts_b200_attend_decode_noalloc ORs them into the caller's). */
#define PTTS_B200_DEVERR_BOUNDS 1u    /* a stream index outside the cache's streams */
#define PTTS_B200_DEVERR_CAPACITY 2u  /* a row's position outside its stream's slots */
#define PTTS_B200_DEVERR_TIMEOUT 4u   /* a bounded wait inside a kernel gave up */
#define PTTS_B200_DEVERR_DUPLICATE 8u /* a stream named by two rows of one decode call */

/* Element types of caches, inputs and outputs. */
#define PTTS_B200_F32 0
#define PTTS_B200_BF16 1

typedef struct ptts_b200_kv ptts_b200_kv;
typedef struct ptts_b200_model ptts_b200_model;
typedef struct ptts_b200_flow ptts_b200_flow; /* the flow head, see "Flow head" below */

/* Shape of a flow-LM transformer: FlowLMConfig (ptts/src/flow_lm.rs:114-146) and the
 * transformer arguments of StreamingTransformer::load (transformer.rs:680-717). */
typedef struct {
    int32_t d_model;          /* 512 */
    int32_t num_heads;        /* 8 (any multiple of 8: 16 in the reference's 1024-wide test config) */
    int32_t num_kv_heads;     /* 8 (grouped-query attention when smaller) */
    int32_t head_dim;         /* 64 */
    int32_t num_layers;       /* 6 (31m) or 9 (40m) */
    int32_t dim_feedforward;  /* 2048 */
    float max_period;         /* RoPE theta, 10000 */
    int32_t gelu;             /* 0: erf (transformer.rs:624), 1: tanh (transformer.rs:500) */
} ptts_b200_config;

/* One layer's weights, HOST pointers, copied to the device by ptts_b200_model_load_layer.
 * Linear weights are int8 [out_features][in_features] with one f32 scale per output row:
 * W = q * scale[row]. Names follow the checkpoint keys (transformer.rs:529-545). */
typedef struct {
    const int8_t* in_proj_host;    /* [(H + 2*KVH)*D][d_model], rows [q | k | v] */
    const float* in_proj_scale_host;
    const int8_t* out_proj_host;   /* [d_model][H*D] */
    const float* out_proj_scale_host;
    const int8_t* linear1_host;    /* [dim_feedforward][d_model] */
    const float* linear1_scale_host;
    const int8_t* linear2_host;    /* [d_model][dim_feedforward] */
    const float* linear2_scale_host;
    const float* norm1_weight_host; /* [d_model] */
    const float* norm1_bias_host;
    const float* norm2_weight_host;
    const float* norm2_bias_host;
} ptts_b200_layer_weights;

/* The message of the last failed call on this thread ("" if none). Borrowed until the next
 * call on this thread. Replaces ptts_last_error (ptts-ffi/include/ptts.h:50). */
const char* ptts_b200_last_error(void);

/* Library version string, e.g. "ptts_b200 0.1 sm_100a". */
const char* ptts_b200_version(void);

/* ---------------------------------------------------------------------------------------
 * KV state: StreamingTransformerState (transformer.rs:328-393) for many streams at once.
 * ------------------------------------------------------------------------------------- */

/* A zero-filled cache of num_layers x num_streams x capacity slots, every length 0.
 * Replaces StreamingMultiheadAttention::init_state (transformer.rs:168-179) and
 * StreamingTransformer::init_state (transformer.rs:731-740). dtype: PTTS_B200_F32 or _BF16. */
int ptts_b200_kv_create(int device, int num_layers, int num_streams, int capacity, int num_heads,
                        int head_dim, int dtype, ptts_b200_kv** out);
void ptts_b200_kv_destroy(ptts_b200_kv* kv);

/* The filled length (current_end) of every stream, from the host-side mirror, no sync. */
int ptts_b200_kv_lengths(const ptts_b200_kv* kv, int32_t* lengths_host);

/* Device pointers of one layer's K and V caches ([H / 8][num_streams][capacity][8][D], see
 * Layouts) and of the device lengths ([num_streams] int32). Borrowed; valid until
 * ptts_b200_kv_destroy. */
int ptts_b200_kv_pointers(const ptts_b200_kv* kv, int layer, void** k, void** v,
                          int32_t** lengths);

/* Count rows[i] more filled positions for stream streams_host[i], on the host mirror and on
 * the device (stream-ordered). StreamingTransformerState::advance (transformer.rs:334-343). */
int ptts_b200_kv_advance(ptts_b200_kv* kv, const int32_t* streams_host, const int32_t* rows_host,
                         int n, void* cuda_stream);

/* Set the lengths of the listed streams (host mirror and device), keeping their slots: rows
 * past the new length are no longer attended and are overwritten by the next appends. The
 * reference lowers current_end the same way when it drops rows (transformer.rs:925). */
int ptts_b200_kv_set_lengths(ptts_b200_kv* kv, const int32_t* streams_host,
                             const int32_t* lengths_host, int n, void* cuda_stream);

/* Set stream lengths to 0 and zero their slots (a fresh session for those streams). */
int ptts_b200_kv_reset(ptts_b200_kv* kv, const int32_t* streams_host, int n, void* cuda_stream);

/* Write `len` rows of K and V (device, [len][H][D], the cache dtype) into slots 0..len of one
 * layer of one stream; with set_length != 0, also set that stream's length to len. The primed
 * voice prefix, as StepGraph loads it (ptts/src/step_graph.rs:291-307). */
int ptts_b200_kv_load_prefix(ptts_b200_kv* kv, int layer, int stream, const void* k,
                             const void* v, int len, int set_length, void* cuda_stream);

/* Copy stream src_stream of `src` into stream dst_stream of `dst` (same layers, heads and
 * dtype, any capacities): the filled prefix is copied, the rest of dst's slots zeroed, dst's
 * length set to src's. Refused with PTTS_B200_ERR_CAPACITY, naming both numbers, when the
 * prefix does not fit. StreamingTransformerState::with_seq_budget (transformer.rs:350-392). */
int ptts_b200_kv_copy_stream(ptts_b200_kv* dst, int dst_stream, const ptts_b200_kv* src,
                             int src_stream, void* cuda_stream);

/* Check the device-side error word that kernels set instead of trapping (bounds, capacity,
 * timeouts of bounded waits). Synchronises the device. Clears the word. */
int ptts_b200_kv_check(ptts_b200_kv* kv);

/* ---- Ring caches: sliding windows (StreamingTransformer::start_ring / set_ring_slot / evict,
 * transformer.rs:840-929) ----------------------------------------------------------------
 * A ring stream keeps every row in the slot it was written to. Its next row goes to the write
 * slot (set_ring_slot), which must not hold a row, at RoPE position = its length; it attends
 * slots 0..max(filled, write + 1) - 1 where a row is held or being written. Evicting hides
 * rows without moving anything, rotates every kept key past `prefix` back by the number of
 * rows evicted (so all distances between kept rows stay) and lowers the length by that many.
 * Ring streams take one row per call, in calls where every sequence has one row (forward,
 * step, attend + kv_advance); prompts, load_prefix, copy_stream and set_lengths refuse them;
 * kv_reset turns them back into appended streams. Refusals leave the cache as it was. */

/* ---- Windowed streams: Mimi's KvCache with a context (transformer.rs:257-317, :395-468) -----
 * A windowed stream's position (its length) grows without bound; position p is stored at slot
 * p % capacity and a query at p attends positions max(0, p - context + 1) .. p (the mask of
 * transformer.rs:762-785, with the cache trimmed to context - 1 rows between calls). A call
 * adds at most capacity - context + 1 rows to it, so no row a query reads is overwritten.
 * Windowed streams run through ptts_b200_attend (+ kv_advance) and through the layer stack's
 * ptts_b200_forward (Mimi's transformer layers); ptts_b200_step, rings, load_prefix and
 * set_lengths refuse them; copy_stream copies them whole into a stream of the same capacity;
 * kv_reset makes them appended streams again. */
int ptts_b200_kv_set_window(ptts_b200_kv* kv, const int32_t* streams_host, int n, int context,
                            void* cuda_stream);

/* Every listed stream becomes a ring: its rows so far stay, the write slot is its length. */
int ptts_b200_kv_start_ring(ptts_b200_kv* kv, const int32_t* streams_host, int n, void* cuda_stream);
/* The slot of a ring stream's next row, 0 <= slot < capacity. */
int ptts_b200_kv_set_ring_slot(ptts_b200_kv* kv, int stream, int slot, void* cuda_stream);
/* set_ring_slot for n ring streams at once: slot slots_host[i] for stream streams_host[i] (no
 * stream twice), in one copy and one launch where n calls of ptts_b200_kv_set_ring_slot take n
 * copies (a batch of sessions sets every ring's slot each frame). The reference sets one
 * state's slot per call (StreamingTransformer::set_ring_slot, transformer.rs:855-872); every
 * entry is checked as there before anything changes. */
int ptts_b200_kv_set_ring_slots(ptts_b200_kv* kv, const int32_t* streams_host, const int32_t* slots_host,
                                int n, void* cuda_stream);
/* Drop the rows in slots[0..n) of a ring stream (each at or past `prefix` and holding a row,
 * no repeats, n at most the length); keys past `prefix` are rotated back by n positions with
 * the RoPE of max_period (RotaryEmbedding::shift_back, rope.rs:26-35), in every layer. */
int ptts_b200_kv_evict(ptts_b200_kv* kv, int stream, int prefix, const int32_t* slots_host, int n,
                       float max_period, void* cuda_stream);

/* ---------------------------------------------------------------------------------------
 * Attention op: the body of StreamingMultiheadAttention::forward after in_proj
 * (transformer.rs:197-248): GQA repeat, RoPE, append, then causal attention.
 * ------------------------------------------------------------------------------------- */

/* For n_seq sequences, sequence i on stream streams_host[i] with rows_host[i] rows:
 * q [n_rows][H][D], k and v [n_rows][KVH][D] (device, in_dtype), rows grouped by sequence in
 * order. Row j of sequence i sits at position p = length[stream] + j: q and k are rotated at p
 * (RotaryEmbedding::forward, rope.rs:81-95, interleaved pairs), k and v are written to slot p
 * of `layer` (complete_kv, transformer.rs:84-91; repeated over the heads sharing a KV head),
 * and the row attends to keys 0..=p (materialize_causal_mask, transformer.rs:94-108; the
 * one-row case is sdpa_decode, transformer.rs:229-230). out [n_rows][H*D] in out_dtype.
 * Lengths are NOT advanced (call ptts_b200_kv_advance after the last layer), as with the
 * device-position step (transformer.rs:822-838). Capacity is checked on the host first. */
int ptts_b200_attend(ptts_b200_kv* kv, int layer, const void* q, const void* k, const void* v,
                     int in_dtype, int num_kv_heads, const int32_t* streams_host,
                     const int32_t* rows_host, int n_seq, float max_period, void* out,
                     int out_dtype, void* cuda_stream);

/* ---------------------------------------------------------------------------------------
 * Quantised linear: Q::LinearQ::forward (transformer.rs:195, :224, :627) for int8 weights with
 * one f32 scale per output row. y[m][n] = scale[n] * sum_k x[m][k] * w[n][k].
 * x [m][k] bf16, w [n][k] int8, scale [n] f32, y [m][n] f32; all device pointers.
 * k and n must be multiples of 64. With n a multiple of 128 it runs on the tcgen05 tensor cores,
 * the int8 weights widened exactly to bf16 on chip and the scale applied to the f32 accumulator:
 * below 4096 rows widened in registers into tensor memory (the MMA's A operand), from 4096 rows
 * on in a persistent kernel that widens them in shared memory. Other n run on the mma.sync
 * kernel.
 * ------------------------------------------------------------------------------------- */
int ptts_b200_linear_i8(int device, const void* x, const int8_t* w, const float* scale, int m,
                        int n, int k, float* y, void* cuda_stream);

/* ---------------------------------------------------------------------------------------
 * Model: StreamingTransformer with int8 per-output-channel linears.
 * ------------------------------------------------------------------------------------- */

/* StreamingTransformer::load (transformer.rs:680-723) minus the file I/O: shapes only, then
 * ptts_b200_model_load_layer for each layer. Refuses head counts that do not divide
 * (transformer.rs:699-707). */
int ptts_b200_model_create(int device, const ptts_b200_config* config, ptts_b200_model** out);
void ptts_b200_model_destroy(ptts_b200_model* model);
/* The shape the model was created with. */
int ptts_b200_model_config(const ptts_b200_model* model, ptts_b200_config* out);
int ptts_b200_model_load_layer(ptts_b200_model* model, int layer,
                               const ptts_b200_layer_weights* weights);

/* A layer from dense f32 linears [out][in] (HOST pointers), e.g. a safetensors checkpoint. The
 * device keeps two f16 planes per linear, f16(W / s) and f16(W / s - hi) with s a power of two
 * per output row: exact to 22 significant bits (every q8_0 weight exactly). Such layers run on
 * the tcgen05 linears at every row count. */
typedef struct {
    const float* in_proj_host;
    const float* out_proj_host;
    const float* linear1_host;
    const float* linear2_host;
    const float* norm1_weight_host;
    const float* norm1_bias_host;
    const float* norm2_weight_host;
    const float* norm2_bias_host;
} ptts_b200_layer_weights_f32;
int ptts_b200_model_load_layer_f32(ptts_b200_model* model, int layer,
                                   const ptts_b200_layer_weights_f32* weights);

/* A layer from GGUF q8_0 linears (the reference's model.q8.gguf, examples/quantize.rs:46-47):
 * each weight [out][in] as rows of in/32 blocks of 34 bytes, an f16 scale d then 32 int8 q,
 * W = q * d (kernels.js:252, :302). Dequantized exactly into the planes above; the layer also
 * keeps q and d / s (s the row's power of two) as f16, from which decode-size calls widen the
 * same weights on chip (the planes when a d / s is not an exact f16). */
typedef struct {
    const void* in_proj_q8_0;
    const void* out_proj_q8_0;
    const void* linear1_q8_0;
    const void* linear2_q8_0;
    const float* norm1_weight_host;
    const float* norm1_bias_host;
    const float* norm2_weight_host;
    const float* norm2_bias_host;
} ptts_b200_layer_weights_q8_0;
int ptts_b200_model_load_layer_q8_0(ptts_b200_model* model, int layer,
                                    const ptts_b200_layer_weights_q8_0* weights);

/* Load a GGUF checkpoint (load_weights, loader.rs:58-67): keys go through the reference's
 * remap_key (loader.rs:15-39: flow_lm.backbone. -> flow_lm.transformer., flow_lm.flow. ->
 * flow_lm.flow_net., ...). Every layer of `model` from flow_lm.transformer.layers.{i}.{self_attn.
 * in_proj, self_attn.out_proj, linear1, linear2}.weight (q8_0, f32, f16 or bf16) and norm1/2;
 * when `flow` is not NULL, every flow-head tensor from flow_lm.<name> and then
 * ptts_b200_flow_finish. Refused, naming the tensor, when one is missing or misshaped. */
int ptts_b200_load_gguf(ptts_b200_model* model, ptts_b200_flow* flow, const char* path);
/* remap_key alone (no device needed): 1 and the new name in `out` (NUL-terminated, at most
 * out_size bytes) when the tensor is kept, 0 when it is dropped, PTTS_B200_ERR_ARG when `out`
 * is too small. */
int ptts_b200_gguf_remap_key(const char* name, char* out, int out_size);

/* The layer scales of StreamingTransformerLayer::forward (transformer.rs:616-618, :632-633;
 * LayerScale::forward, layer_scale.rs:14-16): x += scale1 * attn(LN1 x) and
 * x += scale2 * ff(LN2 x), one factor per channel ([d_model] f32, host). Mimi's layers have
 * them (its transformer is built with a layer_scale); the flow LM's do not. NULL clears one.
 * They are folded into out_proj's and linear2's per-row scales, so a layer reloaded later keeps
 * them. */
int ptts_b200_model_set_layer_scale(ptts_b200_model* model, int layer, const float* scale1_host,
                                    const float* scale2_host);

/* StreamingTransformer::forward (transformer.rs:742-808) for a ragged batch of independent
 * streams: x [n_rows][d_model] bf16 (device) -> y [n_rows][d_model] f32 (device); per layer
 * x += attn(LN1 x); x += W2 GELU(W1 LN2 x). Sequence i is stream streams_host[i] with
 * rows_host[i] rows (a prompt when > 1, a host-position decode step when 1). Lengths advance
 * by rows_host[i] at the end. Windowed streams (ptts_b200_kv_set_window) run Mimi's layers
 * (MimiStreamingMultiheadAttention::forward, transformer.rs:419-468: positions from the
 * stream's absolute offset, keys within the last `context` positions, the mask of
 * transformer.rs:762-785); load such a model with ptts_b200_model_load_layer_f32 and
 * ptts_b200_model_set_layer_scale. */
int ptts_b200_forward(ptts_b200_model* model, ptts_b200_kv* kv, const void* x,
                      const int32_t* streams_host, const int32_t* rows_host, int n_seq, float* y,
                      void* cuda_stream);

/* StreamingTransformer::forward_step (transformer.rs:822-838) with DeviceStep
 * (transformer.rs:111-140): one row per stream for a fixed set of streams whose positions
 * live on the device, replayed as one CUDA graph per stream set. x [n][d_model] bf16 and
 * y [n][d_model] f32 may be device or pinned-host pointers. Lengths advance by one on the
 * device and on the host mirror. The first call for a new stream set records the graph. */
int ptts_b200_step(ptts_b200_model* model, ptts_b200_kv* kv, const int32_t* streams_host, int n,
                   const void* x, float* y, void* cuda_stream);

/* ---------------------------------------------------------------------------------------
 * Decode attention without allocation. No counterpart in the reference: it exists for callers
 * that cannot call cudaMalloc/cudaFree while running (a real-time audio engine that plans every
 * allocation ahead of the frame loop, a server that carves device memory out of its own pool, a
 * host runtime that only hands over raw device pointers).
 *
 * Same arithmetic as ptts_b200_attend with one row per sequence, over a cache the caller owns:
 * k_cache/v_cache [num_streams][capacity][8][64] (one layer, kv_dtype), lengths [num_streams]
 * (device, read and NOT advanced), streams [n] (device), q [n][8][64], k and v [n][KVH][64]
 * (in_dtype), out [n][512] (out_dtype). Row i is rotated at position lengths[streams[i]], its k
 * and v are written to that slot, and it attends to keys 0..=that position.
 *
 * The stream list lives on the device, so the host cannot check it: the kernels do. A row is
 * refused when streams[i] is outside 0..num_streams-1 (err bit PTTS_B200_DEVERR_BOUNDS), when an
 * earlier row names the same stream (PTTS_B200_DEVERR_DUPLICATE; the first row of that stream
 * proceeds), or when its position lengths[streams[i]] is negative or not below `capacity`
 * (PTTS_B200_DEVERR_CAPACITY). A refused row writes no cache row, reads nothing, and its row of
 * `out` is set to zeros. The bits are ORed into *err (a device word the caller clears; may be
 * NULL, in which case a refused row is visible only as its zero output row).
 *
 * Working memory comes from one fixed array in the library (about 4.6 MB per GPU, held until
 * the process exits); n above 1024 is refused with PTTS_B200_ERR_ARG. Every call on a device
 * shares that array, so two calls whose kernels overlap on the GPU (different streams, no
 * ordering between them) race and both results are undefined; order them on one stream. The
 * first call on a device looks the array's address up (cudaGetSymbolAddress) with that device
 * current; make that first call before any stream capture. The address is kept for the rest of
 * the process: do not call this on a device after cudaDeviceReset of that device. No call
 * allocates or frees memory.
 * ------------------------------------------------------------------------------------- */
int ptts_b200_attend_decode_noalloc(void* k_cache, void* v_cache, int num_streams, int capacity,
                                    int kv_dtype, const int32_t* lengths, const int32_t* streams,
                                    int n, const void* q, const void* k, const void* v,
                                    int in_dtype, int num_kv_heads, float max_period, void* out,
                                    int out_dtype, uint32_t* err, void* cuda_stream);

/* Tracing, the counterpart of the reference's `attn` / `transformer-layer` spans
 * (transformer.rs:182, :590), process-wide: while on, ptts_b200_step runs its kernels outside
 * its CUDA graph and ptts_b200_attend (one row per sequence) runs as usual, both with CUDA events
 * around every decode-attention launch and one synchronisation per call. */
typedef struct {
    int64_t steps;            /* traced steps */
    int64_t attn_launches;    /* decode-attention launches timed */
    double attn_ms;           /* their summed device time */
    double attn_bytes;        /* their summed algorithmic bytes: K and V rows read, q read,
                                 output written */
    double step_ms;           /* summed device time of the traced steps */
} ptts_b200_trace;

int ptts_b200_set_tracing(int on);
/* Read (and with reset != 0, clear) the counters. */
int ptts_b200_trace_read(ptts_b200_trace* out, int reset);

/* Kernel timeline of a model's decode steps, taken inside its CUDA graph (where events cannot
 * time single kernels without changing how they overlap). While on, every kernel of the layer
 * stack stamps the GPU's global timer when its first CTA starts, when its first CTA is past its
 * wait on the predecessor kernel, and when its last CTA is done; read returns the launches of
 * the last step, in launch order per lane. A step records a separate graph while stamps are on.
 * max_launches 0 turns stamps off. */
typedef struct {
    char kernel[16];   /* "ln1", "in_proj", "attention", "out_proj", "ln2", "linear1", "linear2",
                          "ln_out" (the last residual reduction) */
    int lane;          /* 0, or 1 for the second lane of a two-lane step */
    int layer;
    double entry_us;   /* first CTA started, from the step's first stamp */
    double start_us;   /* first CTA past its wait on the predecessor */
    double end_us;     /* last CTA done */
    double last_entry_us; /* last CTA started (a late one waited for room on its SM) */
} ptts_b200_stamp;
int ptts_b200_model_stamps(ptts_b200_model* model, int max_launches);
int ptts_b200_model_stamps_read(ptts_b200_model* model, ptts_b200_stamp* out, int max, int* n);

/* ---- Flow head: the rest of a frame -------------------------------------------------------
 * FlowLM's per-frame tail (flow_lm.rs:296-324, :360-410) and its flow net SimpleMLPAdaLN
 * (mlp.rs): out_norm -> EOS logit (out_eos) and the latent from the solver's starting point
 * (LSD: `lsd_steps` Euler steps of the flow net, each conditioned on the times (i/N, (i+1)/N);
 * drifting: one evaluation; pointwise: noise + one evaluation), plus input_linear, which turns
 * the previous latent (or bos_emb) into the next backbone input. z_proj is not supported: the
 * head reads the d_model-wide backbone output (z_dim absent, as in the phonon checkpoints). */

enum { PTTS_B200_FLOW_LSD = 0, PTTS_B200_FLOW_DRIFTING = 1, PTTS_B200_FLOW_POINTWISE = 2 };
enum { PTTS_B200_TIME_RMS = 0, PTTS_B200_TIME_RMS_VAR = 1 };

typedef struct {
    int d_model;     /* backbone width (512); the flow net's cond_channels */
    int flow_dim;    /* flow net width (512), a multiple of 128 */
    int flow_depth;  /* residual blocks (6) */
    int ldim;        /* latent width (32), at most 64 */
    int freq_dim;    /* time embedders' frequency width (256) */
    int flow_type;   /* PTTS_B200_FLOW_* */
    int lsd_steps;   /* LSD solver steps (1) */
    int time_norm;   /* PTTS_B200_TIME_RMS (audiocraft / phonon) or _RMS_VAR (pocket-tts) */
} ptts_b200_flow_config;

/* Weights are set one tensor at a time under the checkpoint's own names (FlowLM::load,
 * flow_lm.rs:196-283, and the SimpleMLPAdaLN paths of mlp.rs), as f32 host arrays of `numel`
 * elements, row-major with Linear weights [out][in]:
 *   input_linear.weight [d_model][ldim]       out_norm.weight, out_norm.bias [d_model]
 *   out_eos.weight [1][d_model], out_eos.bias [1]          bos_emb [ldim]
 *   flow_net.input_proj.{weight [flow_dim][ldim], bias}    flow_net.cond_embed.{weight [flow_dim][d_model], bias}
 *   flow_net.time_embed.{i}.freqs [freq_dim/2]  .mlp.0.{weight [flow_dim][freq_dim], bias}
 *   flow_net.time_embed.{i}.mlp.2.{weight [flow_dim][flow_dim], bias}  .mlp.3.alpha [flow_dim]
 *   flow_net.res_blocks.{i}.in_ln.{weight, bias} [flow_dim]   .mlp.0.{weight, bias}  .mlp.2.{weight, bias}
 *   flow_net.res_blocks.{i}.adaLN_modulation.1.{weight [3 flow_dim][flow_dim], bias}
 *   flow_net.final_layer.adaLN_modulation.1.{weight [2 flow_dim][flow_dim], bias}
 *   flow_net.final_layer.linear.{weight [ldim][flow_dim], bias}
 *   condition [d_model] (optional: the summed condition providers added to every input row)
 * (time_embed.{i} for i < 2 with LSD, none otherwise.) ptts_b200_flow_finish checks that every
 * tensor is present, uploads them (large linears as bf16 hi + lo planes, so f32 weights stay
 * exact to 16 bits) and computes the solver steps' time embeddings once, as FlowLM::load does. */
int ptts_b200_flow_create(int device, const ptts_b200_flow_config* config, ptts_b200_flow** out);
void ptts_b200_flow_destroy(ptts_b200_flow* flow);
int ptts_b200_flow_set_tensor(ptts_b200_flow* flow, const char* name, const float* host, int64_t numel);
int ptts_b200_flow_finish(ptts_b200_flow* flow);

/* FlowLM::sample_from_noise (flow_lm.rs:360-384): t_out [n][d_model] f32 (the backbone output
 * after out_norm), noise [n][ldim] f32 -> latent [n][ldim] f32 and eos [n] f32 (raw logits).
 * Device pointers, stream-ordered. */
int ptts_b200_flow_sample(ptts_b200_flow* flow, const float* t_out, int n, const float* noise,
                          float* latent, float* eos, void* cuda_stream);

/* One frame (FlowLM::sample_next_latent_step, flow_lm.rs:392-410): input_linear(latent) (+
 * condition) as the bf16 backbone input, ptts_b200_step over `streams_host`, out_norm, then
 * ptts_b200_flow_sample. latent_in NULL starts from bos_emb (StepInput::Bos). Device pointers
 * [n][ldim] f32 for latent_in, noise and latent_out, [n] f32 for eos. */
int ptts_b200_frame(ptts_b200_model* model, ptts_b200_flow* flow, ptts_b200_kv* kv,
                    const int32_t* streams_host, int n, const float* latent_in, const float* noise,
                    float* latent_out, float* eos, void* cuda_stream);

#ifdef __cplusplus
}
#endif
#endif
