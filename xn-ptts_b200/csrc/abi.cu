// The C ABI of ptts_b200 (include/ptts_b200.h): objects, argument checks, workspaces, launch
// sequences and the per-stream-set CUDA graph of the device step.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <memory>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "host.h"
#include "kernels.h"
#include "ptts_b200.h"

uint64_t ptts_b200_flow_prepare(ptts_b200_flow* f, int n, int d_model);
int ptts_b200_flow_ldim(const ptts_b200_flow* f);
void ptts_b200_flow_input(ptts_b200_flow* f, const float* latent, __nv_bfloat16* x, int n, cudaStream_t s);
void ptts_b200_flow_head(ptts_b200_flow* f, const float* hidden, int n, const float* noise, float* latent,
                         float* eos, cudaStream_t s, int row_off);

namespace {

using namespace ptts;
using namespace ptts::host;

// Per-call activations of the layer stack (device, sized for `rows` rows).
struct Workspace {
    DevBuf q_rot, h_hi, h_lo, attn_hi, attn_lo, ff_hi, ff_lo, split, part, counters;
    // Prompts of kPersistMinRows+ rows: the current layer's int8 weights widened to f16 (the
    // persistent linears reread every weight tile for each row tile; widening once per call
    // beats widening every tile on chip). Four matrices, 256-byte aligned slices.
    DevBuf wconv;
    void size(const ptts_b200_config& c, int rows) {
        const size_t r = (size_t)rows, hd = (size_t)c.num_heads * c.head_dim;
        q_rot.need(r * hd * 4);
        h_hi.need(r * c.d_model * 2);
        h_lo.need(r * c.d_model * 2);
        attn_hi.need(r * hd * 2);
        attn_lo.need(r * hd * 2);
        ff_hi.need(r * c.dim_feedforward * 2);
        ff_lo.need(r * c.dim_feedforward * 2);
        split.need(4 * r * c.d_model * 4);
        counters.need_zeroed(decode_counter_ints(r) * sizeof(int) * (c.num_heads / kGroupHeads));
    }
};

int sm_count(int dev) {
    int n = 0;
    CK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
    return n;
}

// The decode attention's ring: the compact one for the lanes of a two-lane step (room for a
// linear CTA beside it), else the wide one; PTTS_B200_RING=wide or =compact overrides both.
bool decode_ring_compact(bool lane) {
    static const int force = [] {
        const char* e = getenv("PTTS_B200_RING");
        return !e ? 0 : (e[0] == 'w' ? 1 : (e[0] == 'c' ? 2 : 0));
    }();
    return force == 0 ? lane : force == 2;
}

// CTAs of a split-KV decode launch: one per SM, or for the attention of a two-lane step (which
// shares the SMs with the other lane's linears) PTTS_B200_LANE_CTAS if set (1..SMs). The plan
// and the attention of one launch must use the same count.
int decode_grid(int dev, bool lane) {
    const int sms = sm_count(dev);
    if (!lane) return sms;
    static const int want = [] {
        const char* e = getenv("PTTS_B200_LANE_CTAS");
        return e ? atoi(e) : 0;
    }();
    return want >= 1 && want < sms ? want : sms;
}

void rope_inv_freq(int head_dim, float max_period, float* out) {
    // rope.rs:44-48 with the host libm powf, as the reference computes it.
    const int half = head_dim / 2;
    for (int i = 0; i < half; ++i) out[i] = 1.0f / powf(max_period, (float)i / (float)half);
}

constexpr float kLog2e = 1.4426950408889634f;

// Host-side tile list of the tcgen05 prefill kernels: (first row, rows) per 128 rows of each
// sequence. A tile's work grows with the keys its last row sees (its stream's length before the
// call plus its offset in the sequence), and CTAs start in list order, so the sequences come
// longest first (the short ones fill the last wave instead of a long one starting late), each
// sequence's tiles together and last tile first (they read the same keys, which stay in L2).
std::vector<int2> make_tiles(const std::vector<int32_t>& offsets, const int32_t* streams,
                             const std::vector<int32_t>& h_len) {
    std::vector<std::pair<long long, int>> seqs;  // (keys seen by the last row, sequence)
    for (size_t i = 0; i + 1 < offsets.size(); ++i)
        if (offsets[i + 1] > offsets[i])
            seqs.push_back({(long long)h_len[streams[i]] + offsets[i + 1] - offsets[i], (int)i});
    std::stable_sort(seqs.begin(), seqs.end(),
                     [](const std::pair<long long, int>& x, const std::pair<long long, int>& y) {
                         return x.first > y.first;
                     });
    std::vector<int2> t;
    for (const auto& q : seqs) {
        const int i = q.second, first = offsets[i], end = offsets[i + 1];
        for (int r = first + (end - first - 1) / 128 * 128; r >= first; r -= 128)
            t.push_back(make_int2(r, std::min(128, end - r)));
    }
    return t;
}

// Appends the tile list to a per-call int32 list that goes to the device in one copy, at an
// even index (8-byte aligned on the device, the list's buffer being 256-byte aligned); returns
// that index.
size_t append_tiles(std::vector<int32_t>& packed, const std::vector<int2>& tiles) {
    if (packed.size() % 2) packed.push_back(0);
    const size_t at = packed.size();
    for (const int2& t : tiles) {
        packed.push_back(t.x);
        packed.push_back(t.y);
    }
    return at;
}

bool prefill_on_tensor_cores() {
    const char* e = getenv("PTTS_B200_PREFILL");
    return !(e && e[0] == 'c');  // PTTS_B200_PREFILL=core keeps the CUDA-core kernel
}

// The prompt attention that copies its Q tiles by TMA (attn_prefill_fa.cu), for which the q
// producers (the in_proj epilogue, rope_append) write q as bf16 hi/lo planes; the other prompt
// kernels read f32 q. PTTS_B200_PREFILL=tc1 keeps the one-head-per-CTA tcgen05 kernel.
bool prefill_fa(bool cache_bf16, bool decode, bool windowed) {
    if (decode || !cache_bf16 || windowed || !prefill_on_tensor_cores()) return false;
    const char* e = getenv("PTTS_B200_PREFILL");
    return !(e && e[0] == 't' && e[1] == 'c' && e[2] == '1');
}

// Process-wide tracing of decode-attention launches (ptts_b200_set_tracing).
struct Tracer {
    std::mutex mu;
    bool on = false;
    ptts_b200_trace t{};
};
Tracer& tracer() {
    static Tracer t;
    return t;
}
bool tracing_on() {
    std::lock_guard<std::mutex> g(tracer().mu);
    return tracer().on;
}
void trace_add(int64_t launches, double attn_ms, double attn_bytes, int64_t steps, double step_ms) {
    std::lock_guard<std::mutex> g(tracer().mu);
    tracer().t.attn_launches += launches;
    tracer().t.attn_ms += attn_ms;
    tracer().t.attn_bytes += attn_bytes;
    tracer().t.steps += steps;
    tracer().t.step_ms += step_ms;
}

}  // namespace

struct ptts_b200_kv {
    uint64_t uid;  // distinguishes a new object at a recycled address
    int device, layers, streams, capacity, heads, head_dim, dtype;
    size_t row_bytes;
    DevBuf k, v, len;
    DevBuf err;
    std::vector<int32_t> h_len;
    // Ring streams (start_ring / set_ring_slot / evict, transformer.rs:840-929), on the device
    // and mirrored here: the slot the next row goes to (-1: not a ring), one past the highest
    // slot written, and which slots hold a row attention may see.
    DevBuf ring_write, ring_filled, ring_valid;
    std::vector<int32_t> h_ring_write, h_ring_filled;
    std::vector<uint8_t> h_ring_valid;
    // Windowed streams (Mimi's KvCache, transformer.rs:257-317): the context, 0 = none.
    DevBuf window;
    std::vector<int32_t> h_window;
    // scratch of the attention op
    DevBuf seq_stream, row_offsets, row_stream, row_pos, prefix, part, q_rot, counters;
    Staging staging;
    // What seq_stream holds after the last upload_seq, and on which CUDA stream it was copied: a
    // decode loop that attends and advances the same streams step after step copies the list
    // once, not twice a step (each copy is a DMA round trip between the step's kernels).
    std::vector<int32_t> seq_shadow;
    cudaStream_t seq_shadow_stream = nullptr;
    cudaEvent_t trace_ev[2] = {nullptr, nullptr};
    ~ptts_b200_kv() {
        for (cudaEvent_t e : trace_ev)
            if (e) cudaEventDestroy(e);
    }

    RingArgs ring() const {
        RingArgs r;
        r.write = ring_write.as<int32_t>();
        r.filled = ring_filled.as<int32_t>();
        r.valid = ring_valid.as<uint8_t>();
        r.window = window.as<int32_t>();
        return r;
    }
    bool is_ring(int s) const { return h_ring_write[s] >= 0; }
    // The per-sequence list (streams, then offsets) of an attend or advance call, on the device.
    const int32_t* upload_seq(const std::vector<int32_t>& packed, cudaStream_t s) {
        const size_t n = sizeof(int32_t) * packed.size();
        if (s == seq_shadow_stream && packed == seq_shadow && seq_stream.bytes >= n)
            return seq_stream.as<int32_t>();
        int32_t* d = static_cast<int32_t*>(seq_stream.need(n));
        staging.upload(d, packed.data(), n, s);
        seq_shadow = packed;
        seq_shadow_stream = s;
        return d;
    }
    // Any other list through seq_stream (reset, evict, set_lengths).
    int32_t* upload_scratch(const void* src, size_t n, cudaStream_t s) {
        seq_shadow.clear();
        int32_t* d = static_cast<int32_t*>(seq_stream.need(n));
        staging.upload(d, src, n, s);
        return d;
    }
    bool is_window(int s) const { return h_window[s] > 0; }
    // The host mirror after a row went into stream s's write slot (RingSlots in complete_kv).
    void ring_commit(int s) {
        const int w = h_ring_write[s];
        if (w < 0) return;
        h_ring_valid[(size_t)s * capacity + w] = 1;
        h_ring_filled[s] = std::max(h_ring_filled[s], w + 1);
    }
    // A layer holds its heads in groups of 8 (kv_offset): per group a [streams][capacity] block
    // of rows of 8 heads (group_row_bytes each), groups one after another.
    int groups() const { return heads / kGroupHeads; }
    size_t group_row_bytes() const { return row_bytes / groups(); }
    size_t stream_bytes() const { return (size_t)capacity * group_row_bytes(); }  // in one group
    size_t group_bytes() const { return (size_t)streams * stream_bytes(); }
    size_t layer_bytes() const { return (size_t)groups() * group_bytes(); }
    char* k_layer(int l) const { return k.as<char>() + l * layer_bytes(); }
    char* v_layer(int l) const { return v.as<char>() + l * layer_bytes(); }
    char* k_group(int l, int g) const { return k_layer(l) + g * group_bytes(); }
    char* v_group(int l, int g) const { return v_layer(l) + g * group_bytes(); }
};

// What besides the stream set a recorded step graph depends on: a frame graph also records the
// flow head (its workspace generation) and whether the frame starts from bos_emb.
struct GraphKey {
    uint64_t flow = 0;  // the flow head's identity and workspace generation (0: a plain step)
    bool bos = false;
    bool stamps = false;  // recorded with kernel timeline stamps
    bool operator==(const GraphKey& o) const { return flow == o.flow && bos == o.bos && stamps == o.stamps; }
};

// Kernel timeline of the last step (ptts_b200_model_stamps): four u64 words per launch slot,
// filled by the kernels (stamp_mark), and each slot's kernel, lane and layer.
struct StampLog {
    DevBuf buf;
    int cap = 0, next = 0;
    std::vector<ptts_b200_stamp> meta;
    unsigned long long* words() const { return buf.as<unsigned long long>(); }
    int take(const char* kernel, int lane, int layer) {
        if (next >= cap) return -1;
        ptts_b200_stamp& m = meta[next];
        std::snprintf(m.kernel, sizeof m.kernel, "%s", kernel);
        m.lane = lane;
        m.layer = layer;
        return next++;
    }
};

// One lane of a decode step: rows off .. off + n - 1 of the stream set, with its own row plan
// and workspace so that two lanes can run at the same time.
struct StepLane {
    int off = 0, n = 0;
    DevBuf row_stream, row_pos, prefix;
    Workspace ws;
};

struct StepGraph {
    std::vector<int32_t> streams;
    const ptts_b200_kv* kv = nullptr;
    uint64_t kv_uid = 0;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    DevBuf sid, x, resid;
    StepLane lanes[2];
    int n_lanes = 0;
    GraphKey key;
    DevBuf lat_in, noise, lat_out, eos;  // a frame graph's own inputs and outputs
    ~StepGraph() {
        if (exec) cudaGraphExecDestroy(exec);
        if (graph) cudaGraphDestroy(graph);
    }
};

struct ptts_b200_model {
    int device;
    ptts_b200_config cfg;
    float inv_freq[kMaxPairs];
    struct Layer {
        DevBuf w_qkv, s_qkv, w_out, s_out, w1, s1, w2, s2, ln1g, ln1b, ln2g, ln2b;
        // int8 layers: empty (the tcgen05 linears widen the int8 weights on chip), or with
        // PTTS_B200_WEIGHTS=f16 an exact f16 copy of them that those linears read instead.
        DevBuf h_qkv, h_out, h1, h2;
        // Layers loaded from f32 or q8_0 weights have no int8 copy: h_* hold f16(W / s_row) and
        // l_* the f16 remainders, s_row a power of two per output row (in s_*).
        DevBuf l_qkv, l_out, l1, l2;
        // q8_0 layers also keep their int8 values (q8_*) and block scales divided by the row's
        // power of two (bq_*: [n][k / 32] f16), from which the decode-size linears widen the
        // same hi/lo weights on chip instead of reading the planes (PTTS_B200_Q8=planes: not).
        DevBuf q8_qkv, q8_out, q8_1, q8_2, bq_qkv, bq_out, bq1, bq2;
        // out_proj's and linear2's per-row scales as loaded, and the layer scales (LayerScale,
        // layer_scale.rs:14-16; empty: none) folded into them: s_out = base_out * ls1 and
        // s2 = base_2 * ls2, since ls * (x W^T) = x (ls W)^T row by row.
        std::vector<float> base_out, base_2, ls1, ls2;
        bool loaded = false;
    };
    std::vector<std::unique_ptr<Layer>> layers;
    DevBuf rope;        // RoPE (cos, sin) table [rope_rows][kMaxPairs]
    int rope_rows = 0;
    // forward() workspace
    DevBuf seq_stream, row_stream, row_pos, prefix;
    Workspace ws;
    Staging staging;
    std::unique_ptr<StepGraph> step;
    std::unique_ptr<StepGraph> frame;  // ptts_b200_frame's graph (the step with the flow head)
    cudaStream_t capture_stream = nullptr, lane_stream = nullptr;
    cudaEvent_t lane_start = nullptr, lane_join = nullptr;  // fork / join of a two-lane step
    std::vector<cudaEvent_t> events;  // tracing: [2 * layers] per lane around attention, step start / end
    StampLog stamps;
    ~ptts_b200_model() {
        step.reset();
        frame.reset();
        if (capture_stream) cudaStreamDestroy(capture_stream);
        if (lane_stream) cudaStreamDestroy(lane_stream);
        if (lane_start) cudaEventDestroy(lane_start);
        if (lane_join) cudaEventDestroy(lane_join);
        for (cudaEvent_t e : events) cudaEventDestroy(e);
    }
};

namespace {

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

void check_kv(const ptts_b200_kv* kv) { require(kv != nullptr, PTTS_B200_ERR_ARG, "kv is NULL"); }

void check_launch() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) fail(PTTS_B200_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
}

// Validates sequences against the host mirror; returns total rows, fills offsets.
int check_sequences(const ptts_b200_kv* kv, const int32_t* streams, const int32_t* rows, int n_seq,
                    std::vector<int32_t>& offsets) {
    require(n_seq > 0, PTTS_B200_ERR_ARG, "n_seq must be positive");
    require(streams != nullptr && rows != nullptr, PTTS_B200_ERR_ARG, "streams/rows are NULL");
    offsets.assign(n_seq + 1, 0);
    std::vector<char> seen(kv->streams, 0);
    long long total = 0;
    for (int i = 0; i < n_seq; ++i) {
        const int s = streams[i];
        if (s < 0 || s >= kv->streams)
            fail(PTTS_B200_ERR_ARG,
                 "stream " + std::to_string(s) + " is outside 0.." + std::to_string(kv->streams - 1));
        if (seen[s]) fail(PTTS_B200_ERR_ARG, "stream " + std::to_string(s) + " appears twice");
        seen[s] = 1;
        require(rows[i] >= 1, PTTS_B200_ERR_ARG, "every sequence needs at least one row");
        if (kv->is_ring(s)) {  // StreamingMHAState::complete_kv, transformer.rs:67-73
            if (rows[i] != 1)
                fail(PTTS_B200_ERR_ARG, "a ring cache takes one row at a time, not " + std::to_string(rows[i]) +
                                            " (stream " + std::to_string(s) + ")");
            const int w = kv->h_ring_write[s];
            if (w >= kv->capacity)
                fail(PTTS_B200_ERR_CAPACITY,
                     "ring slot " + std::to_string(w) + " of a " + std::to_string(kv->capacity) + "-slot ring");
            if (kv->h_ring_valid[(size_t)s * kv->capacity + w])
                fail(PTTS_B200_ERR_STATE, "ring slot " + std::to_string(w) +
                                              " still holds a row, evict it first (stream " + std::to_string(s) + ")");
        }
        const long long need = (long long)kv->h_len[s] + rows[i];
        if (kv->is_window(s)) {  // positions grow past the capacity; the window must not wrap
            const int w = kv->h_window[s];      // onto keys the call still reads
            if (rows[i] > kv->capacity - w + 1)
                fail(PTTS_B200_ERR_CAPACITY, "a window of " + std::to_string(w) + " positions over " +
                                                 std::to_string(kv->capacity) + " slots takes at most " +
                                                 std::to_string(kv->capacity - w + 1) + " rows per call, not " +
                                                 std::to_string(rows[i]) + " (stream " + std::to_string(s) + ")");
            require(need < (1LL << 31), PTTS_B200_ERR_CAPACITY, "stream position overflow");
        } else if (need > kv->capacity)
            fail(PTTS_B200_ERR_CAPACITY, "cannot fit " + std::to_string(need) +
                                             " filled KV positions into a budget of " +
                                             std::to_string(kv->capacity) + " (stream " +
                                             std::to_string(s) + ")");
        total += rows[i];
        require(total < (1LL << 30), PTTS_B200_ERR_ARG, "too many rows");
        offsets[i + 1] = (int32_t)total;
    }
    return (int)total;
}

// A call with a prompt (some sequence of more than one row) plans rows by position; a ring
// stream's row must go to its write slot, so ring streams only join all-decode calls.
// Keys the next decode row of stream st attends (the decode plan's count; tracing only).
long long attended_keys(const ptts_b200_kv* kv, int st) {
    const long long len = kv->h_len[st];
    if (kv->is_window(st)) return std::min<long long>(len + 1, kv->h_window[st]);
    if (kv->is_ring(st)) return std::max<long long>(kv->h_ring_filled[st], kv->h_ring_write[st] + 1);
    return len + 1;
}

// Windowed streams (Mimi) run through ptts_b200_forward and the attention op, not the device
// step: like the reference's, whose device-position step runs flow-LM attention only
// (transformer.rs:603-605).
void refuse_window(const ptts_b200_kv* kv, const int32_t* streams, int n) {
    for (int i = 0; i < n; ++i)
        if (kv->is_window(streams[i]))
            fail(PTTS_B200_ERR_UNSUPPORTED,
                 "stream " + std::to_string(streams[i]) +
                     " is windowed: windowed streams run through ptts_b200_forward or ptts_b200_attend, "
                     "not the device step");
}

void refuse_ring_prompt(const ptts_b200_kv* kv, const int32_t* streams, int n, bool decode) {
    if (decode) return;
    for (int i = 0; i < n; ++i)
        if (kv->is_ring(streams[i]))
            fail(PTTS_B200_ERR_ARG,
                 "a ring cache takes one row at a time, in calls where every sequence has one row (stream " +
                     std::to_string(streams[i]) + ")");
}

// Ring state of stream st back to "not a ring" (kv_reset).
void ring_clear(ptts_b200_kv* kv, int st, cudaStream_t s) {
    kv->h_ring_write[st] = -1;
    kv->h_ring_filled[st] = 0;
    std::fill(kv->h_ring_valid.begin() + (size_t)st * kv->capacity,
              kv->h_ring_valid.begin() + (size_t)(st + 1) * kv->capacity, 0);
    const int32_t wf[2] = {-1, 0};
    kv->staging.upload(kv->ring_write.as<int32_t>() + st, &wf[0], sizeof(int32_t), s);
    kv->staging.upload(kv->ring_filled.as<int32_t>() + st, &wf[1], sizeof(int32_t), s);
    CK(cudaMemsetAsync(kv->ring_valid.as<uint8_t>() + (size_t)st * kv->capacity, 0, kv->capacity, s));
}

// Decode (every sequence one row) or ragged plan into the given buffers; `row_pos` holds the
// positions and then the slots.
RowPlan make_plan(const ptts_b200_kv* kv, bool decode, const int32_t* d_seq_stream,
                  const int32_t* d_row_offsets, int n_seq, int n_rows, DevBuf& row_stream,
                  DevBuf& row_pos, DevBuf& prefix, cudaStream_t s) {
    RowPlan plan;
    plan.row_stream = static_cast<int32_t*>(row_stream.need(sizeof(int32_t) * n_rows));
    plan.row_pos = static_cast<int32_t*>(row_pos.need(2 * sizeof(int32_t) * n_rows));
    plan.row_slot = plan.row_pos + n_rows;
    plan.prefix = static_cast<int32_t*>(prefix.need(sizeof(int32_t) * (n_rows + 1 + kMaxDecodeGrid)));
    plan.cta_first = plan.prefix + n_rows + 1;
    if (decode)
        launch_plan_decode(kv->len.as<int32_t>(), d_seq_stream, n_seq, kv->streams, kv->capacity,
                           plan, kv->ring(), sm_count(kv->device), kv->err.as<uint32_t>(), s);
    else
        launch_plan_rows(kv->len.as<int32_t>(), d_seq_stream, d_row_offsets, n_seq, n_rows,
                         kv->streams, kv->capacity, plan, kv->window.as<int32_t>(), kv->err.as<uint32_t>(), s);
    return plan;
}

// Tiles of a prefill call (device list + count); empty for decode calls.
struct Tiles {
    const int2* dev = nullptr;
    int n = 0;
    bool windowed = false;  // a windowed stream is in the call: the CUDA-core kernel maps its slots
};

// The attention of head group g (heads 8g .. 8g + 7) on its cache block and its columns of q_rot
// and out (rows of ld = H * 64 elements): one launch.
void attention_group(const ptts_b200_kv* kv, int layer, int g, bool decode, const RowPlan& plan, int n_rows,
                     const float* q_rot, void* out, void* out_lo, int out_mode, DevBuf& part, DevBuf& counters,
                     const Tiles& tiles, cudaStream_t s, bool compact, unsigned long long* stamps, int stamp) {
    const bool bf16 = kv->dtype == PTTS_B200_BF16;
    const float qscale = (1.0f / sqrtf((float)kv->head_dim)) * kLog2e;  // transformer.rs:215
    const int ld = kv->heads * kHeadDim, G = kv->groups();
    const size_t col = (size_t)g * kRowWidth, out_elem = out_mode == kOutF32 ? 4 : 2;
    void* o = static_cast<char*>(out) + col * out_elem;
    void* o_lo = out_lo ? static_cast<char*>(out_lo) + col * out_elem : nullptr;
    if (decode) {
        const int grid = decode_grid(kv->device, compact);
        // Partial records and merge counters: a slice per group.
        const size_t n_part = decode_part_floats(n_rows, grid), n_cnt = decode_counter_ints(n_rows);
        DecodeArgs a{};
        a.k_cache = kv->k_group(layer, g);
        a.v_cache = kv->v_group(layer, g);
        a.stream_bytes = (long long)kv->stream_bytes();
        a.row_stream = plan.row_stream;
        a.prefix = plan.prefix;
        a.q = q_rot + col;
        a.out = o;
        a.out_lo = o_lo;
        a.out_mode = out_mode;
        a.ld = ld;
        a.part = static_cast<float*>(part.need(sizeof(float) * n_part * G)) + n_part * g;
        a.counters = static_cast<int*>(counters.need_zeroed(sizeof(int) * n_cnt * G)) + n_cnt * g;
        a.cta_first = plan.cta_first;
        a.B = n_rows;
        a.qscale = qscale;
        a.err = kv->err.as<uint32_t>();
        a.ring_write = kv->ring_write.as<int32_t>();
        a.ring_valid = kv->ring_valid.as<uint8_t>();
        a.capacity = kv->capacity;
        a.window = kv->window.as<int32_t>();
        a.row_pos = plan.row_pos;
        // The in_proj or rope_append launch (or, past group 0, the previous group's attention,
        // which runs only after it) sits between the plan and this one.
        a.prestart = true;
        a.stamps = stamps;
        a.stamp = stamp;
        launch_decode_attn(a, bf16, grid, s, decode_ring_compact(compact));
    } else {
        PrefillArgs a{};
        a.k_cache = kv->k_group(layer, g);
        a.v_cache = kv->v_group(layer, g);
        a.stream_elems = (long long)kv->capacity * kRowWidth;
        a.row_stream = plan.row_stream;
        a.row_pos = plan.row_pos;
        a.window = kv->window.as<int32_t>();
        a.q = q_rot + col;
        a.out = o;
        a.out_lo = o_lo;
        a.out_mode = out_mode;
        a.ld = ld;
        a.rows = n_rows;
        a.qscale = qscale;
        a.err = kv->err.as<uint32_t>();
        if (tiles.n > 0 && prefill_fa(bf16, decode, tiles.windowed)) {
            // The head-group pipeline (attn_prefill_fa.cu), Q tiles by TMA from the hi/lo planes.
            a.q = nullptr;
            a.q_hi = reinterpret_cast<const __nv_bfloat16*>(q_rot) + col;
            a.q_lo = reinterpret_cast<const __nv_bfloat16*>(q_rot) + (size_t)n_rows * ld + col;
            require(launch_prefill_attn_fa(a, tiles.dev, tiles.n, kv->streams, kv->capacity, s), PTTS_B200_ERR_CUDA,
                    "could not describe the prompt attention's tensors (cuTensorMapEncodeTiled)");
        } else if (bf16 && tiles.n > 0 && prefill_on_tensor_cores() && !tiles.windowed) {
            launch_prefill_attn_tc(a, tiles.dev, tiles.n, s);
        } else {
            launch_prefill_attn(a, bf16, s);
        }
    }
    check_launch();
}

// q_rot is the rotated q: f32 [n_rows][H * 64], or for prompts where prefill_fa holds, its bf16
// hi plane followed by the lo plane (n_rows x H * 64 each). One launch per group of 8 heads.
void attention(const ptts_b200_kv* kv, int layer, bool decode, const RowPlan& plan, int n_rows,
               const float* q_rot, void* out, void* out_lo, int out_mode, DevBuf& part,
               DevBuf& counters, const Tiles& tiles, cudaStream_t s, bool compact = false,
               unsigned long long* stamps = nullptr, int stamp = -1) {
    for (int g = 0; g < kv->groups(); ++g)
        attention_group(kv, layer, g, decode, plan, n_rows, q_rot, out, out_lo, out_mode, part, counters, tiles, s,
                        compact, stamps, g == 0 ? stamp : -1);
}

void check_model_kv(const ptts_b200_model* m, const ptts_b200_kv* kv) {
    require(m != nullptr, PTTS_B200_ERR_ARG, "model is NULL");
    check_kv(kv);
    require(m->device == kv->device, PTTS_B200_ERR_STATE, "model and kv live on different devices");
    require(kv->layers == m->cfg.num_layers, PTTS_B200_ERR_STATE,
            "kv has " + std::to_string(kv->layers) + " layers, the model " +
                std::to_string(m->cfg.num_layers));
    require(kv->heads == m->cfg.num_heads && kv->head_dim == m->cfg.head_dim, PTTS_B200_ERR_STATE,
            "kv heads/head_dim differ from the model's");
    require(kv->dtype == PTTS_B200_BF16, PTTS_B200_ERR_UNSUPPORTED,
            "the model runs on a bf16 KV cache");
    for (int l = 0; l < m->cfg.num_layers; ++l)
        require(m->layers[l]->loaded, PTTS_B200_ERR_STATE,
                "layer " + std::to_string(l) + " has no weights (ptts_b200_model_load_layer)");
}

// Split-K slices of out_proj and linear2 at a row count: enough CTAs to fill the GPU at decode
// sizes, none for prompts; K / splits stays a multiple of 64.
int split_for(int rows, int k, int want) {
    if (rows >= 1024) return 1;
    int sp = want;
    while (sp > 1 && (k % sp != 0 || (k / sp) % 64 != 0)) sp /= 2;
    return sp;
}

// Whether decode-size linears of q8_0 layers widen the block-scaled int8 values on chip
// (default) or read the f16 planes (PTTS_B200_Q8=planes).
bool q8_on_chip() {
    const char* e = getenv("PTTS_B200_Q8");
    return !(e && e[0] == 'p');
}

// StreamingTransformer::forward / forward_step body (transformer.rs:591-634 for every layer):
//   LN1 (+ previous layer's split-K slices) -> in_proj (RoPE + append) -> attention ->
//   out_proj (split-K) -> LN2 (+ slices) -> linear1 + GELU -> linear2 (split-K),
// then a last reduction into the residual. x_in (bf16) seeds the f32 residual `resid`.
// `lane`: this is one of two lanes of a decode step running side by side; the attention takes
// its compact ring, and `after_qkv0` (if set) is recorded once the first in_proj is launched.
struct LaneOpts {
    int id = 0;
    bool lane = false;
    cudaEvent_t after_qkv0 = nullptr;
    StampLog* stamps = nullptr;  // kernel timeline, or none
};
void run_layers(const ptts_b200_model* m, const ptts_b200_kv* kv, bool decode, const RowPlan& plan,
                int rows, const __nv_bfloat16* x_in, float* resid, Workspace& w, cudaStream_t s,
                cudaEvent_t* attn_ev = nullptr, const Tiles& tiles = Tiles{}, const LaneOpts& lo = LaneOpts{}) {
    const ptts_b200_config& c = m->cfg;
    const int hd = c.num_heads * c.head_dim;
    const int nqkv = hd + 2 * c.num_kv_heads * c.head_dim;
    const int s_out = split_for(rows, hd, 4), s_ff2 = split_for(rows, c.dim_feedforward, 4);
    uint32_t* err = kv->err.as<uint32_t>();
    auto* h_hi = w.h_hi.as<__half>();
    auto* h_lo = w.h_lo.as<__half>();
    auto* split = w.split.as<float>();
    int pending = 0;  // split-K slices not yet added to the residual
    int layer = 0;
    // A timeline slot for the next launch, when stamps are on.
    auto stamp = [&](auto& args, const char* kernel) {
        if (!lo.stamps) return;
        args.stamps = lo.stamps->words();
        args.stamp = lo.stamps->take(kernel, lo.id, layer);
    };
    auto ln = [&](const float* g, const float* b, const __nv_bfloat16* x_bf16, bool normalise, const char* name) {
        LnArgs a{};
        a.M = rows;
        a.d = c.d_model;
        a.resid = resid;
        a.x_bf16 = x_bf16;
        a.part = split;
        a.nsplit = pending;
        a.gamma = g;
        a.beta = b;
        a.hi = normalise ? h_hi : nullptr;
        a.lo = normalise ? h_lo : nullptr;
        stamp(a, name);
        launch_ln(a, s);
        check_launch();
        pending = 0;
    };
    // The weight fields of a linear: the q8_0 on-chip form at decode sizes (q8 set per layer),
    // else the int8 values or the 16-bit planes.
    bool q8 = false;
    auto set_weights = [&](LinearArgs& x, const DevBuf& wq, const void* wh, const DevBuf& wl, const DevBuf& q8v,
                           const DevBuf& bq) {
        if (q8) {
            x.w = q8v.as<int8_t>();
            x.wblk = bq.as<__half>();
        } else {
            x.w = wq.as<int8_t>();
            x.wh = wh;
            x.wh_lo = wl.p;
        }
    };
    auto residual_gemm = [&](const void* a_hi, const void* a_lo, const DevBuf& wq, const void* wh,
                             const DevBuf& wl, const DevBuf& q8v, const DevBuf& bq, const DevBuf& sc, int k,
                             int splits) {
        LinearArgs o{};
        o.M = rows;
        o.N = c.d_model;
        o.K = k;
        o.splits = splits;
        o.a = a_hi;
        o.a_lo = a_lo;
        set_weights(o, wq, wh, wl, q8v, bq);
        o.scale = sc.as<float>();
        o.y = splits > 1 ? split : resid;
        o.err = err;
        stamp(o, k == c.d_model ? "out_proj" : "linear2");
        require(launch_linear(o, splits > 1 ? EPI_PARTIAL : EPI_RESID, s), PTTS_B200_ERR_UNSUPPORTED,
                "no kernel for this linear's shape");
        check_launch();
        if (splits > 1) pending = splits;
    };
    // Prompt-size calls on int8 layers read their weights widened once per layer (see wconv).
    // Prompts only: decode steps are recorded into graphs, where the workspace cannot grow.
    const bool widen = !decode && rows >= kPersistMinRows && s_out == 1 && s_ff2 == 1;
    const size_t n_qkv = (size_t)nqkv * c.d_model, n_out = (size_t)c.d_model * hd;
    const size_t n_ff1 = (size_t)c.dim_feedforward * c.d_model, n_ff2 = n_ff1;
    auto al = [](size_t bytes) { return (bytes + 255) / 256 * 256; };
    const size_t o_out = al(2 * n_qkv), o_ff1 = o_out + al(2 * n_out), o_ff2 = o_ff1 + al(2 * n_ff1);
    for (int l = 0; l < c.num_layers; ++l) {
        layer = l;
        const auto& L = *m->layers[l];
        q8 = rows < kPersistMinRows && L.bq_qkv.p && q8_on_chip();
        // Per-linear 16-bit weights: the layer's own planes, the widened prompt copy, or none.
        const void *wh_qkv = L.h_qkv.p, *wh_out = L.h_out.p, *wh_1 = L.h1.p, *wh_2 = L.h2.p;
        if (widen && L.w_qkv.p && !L.h_qkv.p) {
            unsigned char* base = static_cast<unsigned char*>(w.wconv.need(o_ff2 + al(2 * n_ff2)));
            I8Widen wd;
            const DevBuf* src[4] = {&L.w_qkv, &L.w_out, &L.w1, &L.w2};
            const size_t off[4] = {0, o_out, o_ff1, o_ff2}, n[4] = {n_qkv, n_out, n_ff1, n_ff2};
            for (int i = 0; i < 4; ++i) {
                wd.src[i] = src[i]->as<int8_t>();
                wd.dst[i] = reinterpret_cast<__half*>(base + off[i]);
                wd.n[i] = (long long)n[i];
            }
            launch_widen_i8(wd, s);
            check_launch();
            wh_qkv = wd.dst[0];
            wh_out = wd.dst[1];
            wh_1 = wd.dst[2];
            wh_2 = wd.dst[3];
        }
        ln(L.ln1g.as<float>(), L.ln1b.as<float>(), l == 0 ? x_in : nullptr, true, "ln1");
        // in_proj, RoPE + append epilogue
        LinearArgs a{};
        a.M = rows;
        a.N = nqkv;
        a.K = c.d_model;
        a.a = h_hi;
        a.a_lo = h_lo;
        set_weights(a, L.w_qkv, wh_qkv, L.l_qkv, L.q8_qkv, L.bq_qkv);
        a.scale = L.s_qkv.as<float>();
        a.yq = w.q_rot.as<float>();
        if (prefill_fa(kv->dtype == PTTS_B200_BF16, decode, tiles.windowed) && tiles.n > 0) {
            a.yq_hi = w.q_rot.as<__nv_bfloat16>();  // two bf16 planes in the f32 buffer's bytes
            a.yq_lo = a.yq_hi + (size_t)rows * hd;
            a.yq_scale = (1.0f / sqrtf((float)c.head_dim)) * kLog2e;  // transformer.rs:215, exp2 domain
        }
        a.row_stream = plan.row_stream;
        a.row_pos = plan.row_pos;
        a.row_slot = plan.row_slot;
        a.k_cache = reinterpret_cast<__nv_bfloat16*>(kv->k_layer(l));
        a.v_cache = reinterpret_cast<__nv_bfloat16*>(kv->v_layer(l));
        a.heads = c.num_heads;
        a.kv_heads = c.num_kv_heads;
        a.num_streams = kv->streams;
        a.capacity = kv->capacity;
        require(m->rope_rows >= kv->capacity, PTTS_B200_ERR_STATE, "RoPE table shorter than the cache");
        a.rope = m->rope.as<float2>();
        a.rope_rows = m->rope_rows;
        a.err = err;
        stamp(a, "in_proj");
        require(launch_linear(a, EPI_QKV, s), PTTS_B200_ERR_UNSUPPORTED, "no kernel for in_proj's shape");
        check_launch();
        if (l == 0 && lo.after_qkv0) CK(cudaEventRecord(lo.after_qkv0, s));
        // attention over the cache
        if (attn_ev) CK(cudaEventRecord(attn_ev[2 * l], s));
        DecodeArgs stamped;  // carries the attention's timeline slot
        stamp(stamped, "attention");
        attention(kv, l, decode, plan, rows, w.q_rot.as<float>(), w.attn_hi.p, w.attn_lo.p,
                  kOutHiLo, w.part, w.counters, tiles, s, lo.lane, stamped.stamps, stamped.stamp);
        if (attn_ev) CK(cudaEventRecord(attn_ev[2 * l + 1], s));
        // out_proj + residual
        residual_gemm(w.attn_hi.as<__half>(), w.attn_lo.as<__half>(), L.w_out, wh_out, L.l_out, L.q8_out,
                      L.bq_out, L.s_out, hd, s_out);
        // LN2, linear1 + GELU
        ln(L.ln2g.as<float>(), L.ln2b.as<float>(), nullptr, true, "ln2");
        LinearArgs f1{};
        f1.M = rows;
        f1.N = c.dim_feedforward;
        f1.K = c.d_model;
        f1.a = h_hi;
        f1.a_lo = h_lo;
        set_weights(f1, L.w1, wh_1, L.l1, L.q8_1, L.bq1);
        f1.scale = L.s1.as<float>();
        f1.yb = w.ff_hi.as<__half>();
        f1.yb_lo = w.ff_lo.as<__half>();
        f1.gelu_tanh = c.gelu;
        f1.err = err;
        stamp(f1, "linear1");
        require(launch_linear(f1, EPI_GELU, s), PTTS_B200_ERR_UNSUPPORTED, "no kernel for linear1's shape");
        check_launch();
        // linear2 + residual
        residual_gemm(w.ff_hi.as<__half>(), w.ff_lo.as<__half>(), L.w2, wh_2, L.l2, L.q8_2, L.bq2, L.s2,
                      c.dim_feedforward, s_ff2);
    }
    if (pending) ln(nullptr, nullptr, nullptr, false, "ln_out");
}

// Grows the RoPE table to `rows` positions. A captured step graph holds the old table's address,
// so it is dropped when the table moves.
void ensure_rope(ptts_b200_model* m, int rows, cudaStream_t s) {
    if (m->rope_rows >= rows) return;
    // Grown geometrically (windowed streams ask for one more position every frame).
    if (m->rope_rows > 0) rows = std::max(rows, std::min(2 * m->rope_rows, m->rope_rows + (1 << 20)));
    CK(cudaStreamSynchronize(s));
    m->step.reset();
    m->frame.reset();
    RopeFreqs f;
    std::memcpy(f.inv_freq, m->inv_freq, sizeof(f.inv_freq));
    launch_rope_table(f, static_cast<float2*>(m->rope.need(sizeof(float2) * kMaxPairs * (size_t)rows)), rows, s);
    check_launch();
    m->rope_rows = rows;
}

// f32 -> f16 bits, round to nearest even, subnormals included (|x| <= 65504 here).
uint16_t f16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    const uint32_t sign = (u >> 16) & 0x8000u;
    const int exp = (int)((u >> 23) & 0xFF) - 127 + 15;
    uint32_t man = u & 0x7FFFFFu;
    if (((u >> 23) & 0xFF) == 0) return (uint16_t)sign;  // f32 zero or subnormal -> 0
    if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
    if (exp <= 0) {  // f16 subnormal: value = man16 * 2^-24
        if (exp < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int shift = 14 - exp;  // bits dropped from the 24-bit significand
        uint32_t q = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (q & 1u))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t q = ((uint32_t)exp << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) ++q;  // may carry into the exponent
    return (uint16_t)(sign | q);
}
// A linear of f32 weights [n][k] as f16 planes: hi = f16(W / s), lo = f16(W / s - hi) with
// s = 2^ceil(log2(max |W_row|)) per row, so W/s is exact to 22 significant bits for weights
// within 2^-14 of their row's largest (q8_0 weights, 18 bits, are exact); lo is dropped when it
// is all zero.
std::vector<float> upload_dense(DevBuf& hi, DevBuf& lo, DevBuf& scale, const float* w, size_t n, size_t k) {
    std::vector<uint16_t> h(n * k), l(n * k);
    std::vector<float> sc(n);
    bool any_lo = false;
    for (size_t r = 0; r < n; ++r) {
        float amax = 0.f;
        for (size_t c = 0; c < k; ++c) amax = std::max(amax, std::fabs(w[r * k + c]));
        require(std::isfinite(amax), PTTS_B200_ERR_ARG, "a weight is not finite");
        int e = 0;
        if (amax > 0.f) std::frexp(amax, &e);  // amax = f * 2^e, 0.5 <= f < 1
        sc[r] = std::ldexp(1.0f, e);
        for (size_t c = 0; c < k; ++c) {
            const float x = std::ldexp(w[r * k + c], -e);
            h[r * k + c] = f16_bits(x);
            l[r * k + c] = f16_bits(x - f16_value(h[r * k + c]));
            any_lo = any_lo || (l[r * k + c] & 0x7FFFu) != 0;
        }
    }
    CK(cudaMemcpy(hi.need(n * k * 2), h.data(), n * k * 2, cudaMemcpyHostToDevice));
    if (any_lo) CK(cudaMemcpy(lo.need(n * k * 2), l.data(), n * k * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(scale.need(n * 4), sc.data(), n * 4, cudaMemcpyHostToDevice));
    return sc;
}

// Uploads out_proj's and linear2's effective row scales: the loaded ones times the layer scales.
void apply_layer_scale(ptts_b200_model::Layer& L) {
    auto put = [](DevBuf& dst, const std::vector<float>& base, const std::vector<float>& ls) {
        if (base.empty()) return;
        std::vector<float> e(base);
        if (!ls.empty())
            for (size_t i = 0; i < e.size(); ++i) e[i] *= ls[i];
        CK(cudaMemcpy(dst.need(e.size() * 4), e.data(), e.size() * 4, cudaMemcpyHostToDevice));
    };
    put(L.s_out, L.base_out, L.ls1);
    put(L.s2, L.base_2, L.ls2);
}

// GGUF q8_0 blocks (34 bytes: f16 d, then 32 int8 q) of an [n][k] weight -> f32 W = q * d.
std::vector<float> dequant_q8_0(const void* blocks, size_t n, size_t k) {
    std::vector<float> w(n * k);
    const unsigned char* b = static_cast<const unsigned char*>(blocks);
    for (size_t i = 0; i < n * k / 32; ++i, b += 34) {
        uint16_t d16;
        std::memcpy(&d16, b, 2);
        const float d = f16_value(d16);
        for (int j = 0; j < 32; ++j) w[i * 32 + j] = (float)(int8_t)b[2 + j] * d;
    }
    return w;
}

// A q8_0 linear's values (int8 [n][k]) and its block scales d over the row's power of two 2^e
// (upload_dense's row scale for the same weights: e from the row's largest |q d|), [n][k / 32]
// f16: q * (d 2^-e) is exactly the value the row's f16 hi/lo planes split. False (nothing
// uploaded) when a scale d 2^-e is not exact in f16 (a block 2^14 and more below its row's
// largest): the kernel's f16 arithmetic then could not reproduce the planes.
bool upload_q8_blocks(DevBuf& q8, DevBuf& bq, const void* blocks, const float* w, size_t n, size_t k) {
    std::vector<int8_t> q(n * k);
    std::vector<uint16_t> d(n * k / 32);
    const unsigned char* b = static_cast<const unsigned char*>(blocks);
    for (size_t r = 0; r < n; ++r) {
        float amax = 0.f;
        for (size_t c = 0; c < k; ++c) amax = std::max(amax, std::fabs(w[r * k + c]));
        int e = 0;
        if (amax > 0.f) std::frexp(amax, &e);
        for (size_t blk = 0; blk < k / 32; ++blk) {
            const unsigned char* p = b + (r * (k / 32) + blk) * 34;
            uint16_t d16;
            std::memcpy(&d16, p, 2);
            const float ds = std::ldexp(f16_value(d16), -e);
            d[r * (k / 32) + blk] = f16_bits(ds);
            if (f16_value(d[r * (k / 32) + blk]) != ds) return false;
            std::memcpy(&q[r * k + blk * 32], p + 2, 32);
        }
    }
    CK(cudaMemcpy(q8.need(q.size()), q.data(), q.size(), cudaMemcpyHostToDevice));
    CK(cudaMemcpy(bq.need(d.size() * 2), d.data(), d.size() * 2, cudaMemcpyHostToDevice));
    return true;
}

// A layer from f32 linears: the f16 planes above, no int8 copy.
void load_dense_layer(ptts_b200_model* model, int layer, const float* in_proj, const float* out_proj,
                      const float* linear1, const float* linear2, const float* n1w, const float* n1b,
                      const float* n2w, const float* n2b) {
    require(layer >= 0 && layer < model->cfg.num_layers, PTTS_B200_ERR_ARG, "layer out of range");
    require(in_proj && out_proj && linear1 && linear2 && n1w && n1b && n2w && n2b, PTTS_B200_ERR_ARG,
            "a weight pointer is NULL");
    const ptts_b200_config& c = model->cfg;
    const size_t dm = c.d_model, hd = (size_t)c.num_heads * c.head_dim;
    const size_t nqkv = hd + 2 * (size_t)c.num_kv_heads * c.head_dim, ff = c.dim_feedforward;
    DeviceScope scope(model->device);
    auto& L = *model->layers[layer];
    for (DevBuf* b : {&L.w_qkv, &L.w_out, &L.w1, &L.w2, &L.l_qkv, &L.l_out, &L.l1, &L.l2, &L.q8_qkv, &L.q8_out,
                      &L.q8_1, &L.q8_2, &L.bq_qkv, &L.bq_out, &L.bq1, &L.bq2})
        b->release();
    upload_dense(L.h_qkv, L.l_qkv, L.s_qkv, in_proj, nqkv, dm);
    L.base_out = upload_dense(L.h_out, L.l_out, L.s_out, out_proj, dm, hd);
    upload_dense(L.h1, L.l1, L.s1, linear1, ff, dm);
    L.base_2 = upload_dense(L.h2, L.l2, L.s2, linear2, dm, ff);
    auto put = [](DevBuf& b, const void* src, size_t n) { CK(cudaMemcpy(b.need(n), src, n, cudaMemcpyHostToDevice)); };
    put(L.ln1g, n1w, dm * 4);
    put(L.ln1b, n1b, dm * 4);
    put(L.ln2g, n2w, dm * 4);
    put(L.ln2b, n2b, dm * 4);
    apply_layer_scale(L);
    CK(cudaDeviceSynchronize());
    L.loaded = true;
}

bool is_device_pointer(const void* p) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged;
}

}  // namespace

// How many lanes a decode step of n rows runs in. Two lanes (two halves of the stream set on two
// streams inside the graph) let one half's latency-bound linears run beside the other half's
// HBM-bound attention; below 128 rows a step runs as one. PTTS_B200_LANES=1 keeps one lane.
int step_lanes(int n) {
    static const bool one = [] {
        const char* e = getenv("PTTS_B200_LANES");
        return e && e[0] == '1';
    }();
    return (!one && n >= 128) ? 2 : 1;
}

// One decode step of the stack for `streams` (transformer.rs:822-838 with DeviceStep), recorded
// once per stream set as a CUDA graph in `slot` and replayed: `inputs` fills the graph's input
// buffers (before the replay), `pre` launches extra kernels before the layers and `post(stream,
// row_off, rows)` after each lane's layers, on that lane's stream, inside the recorded body.
// With tracing on, the body runs un-recorded on one stream (the lanes one after the other),
// timed per attention.
//
// Two lanes: rows [0, n0) run on the capture stream, rows [n0, n) on a second stream forked
// from it. The second lane starts once the first has launched its first in_proj, so the first
// lane's attention meets the second lane's linears; both join before `post`.
template <class Inputs, class Pre, class Post>
void run_step(ptts_b200_model* model, ptts_b200_kv* kv, const int32_t* streams_host, int n,
              std::unique_ptr<StepGraph>& slot, const GraphKey& key, cudaStream_t s, Inputs&& inputs,
              Pre&& pre, Post&& post) {
    std::vector<int32_t> ones(n > 0 ? n : 0, 1), offsets;
    check_sequences(kv, streams_host, ones.data(), n, offsets);  // capacity for one more row
    refuse_window(kv, streams_host, n);
    const ptts_b200_config& c = model->cfg;
    ensure_rope(model, kv->capacity, s);
    const int n_lanes = step_lanes(n);
    const int grid = decode_grid(kv->device, n_lanes > 1);
    GraphKey gkey = key;
    gkey.stamps = model->stamps.cap > 0;
    StepGraph* g = slot.get();
    const bool same = g && g->kv == kv && g->kv_uid == kv->uid && g->key == gkey && g->streams.size() == (size_t)n &&
                      g->n_lanes == n_lanes &&
                      std::memcmp(g->streams.data(), streams_host, sizeof(int32_t) * n) == 0;
    if (!same) {
        // Buffers of this stream set.
        CK(cudaStreamSynchronize(s));
        slot.reset();
        auto ng = std::make_unique<StepGraph>();
        ng->streams.assign(streams_host, streams_host + n);
        ng->kv = kv;
        ng->kv_uid = kv->uid;
        ng->key = gkey;
        int32_t* sid = static_cast<int32_t*>(ng->sid.need(sizeof(int32_t) * n));
        CK(cudaMemcpy(sid, streams_host, sizeof(int32_t) * n, cudaMemcpyHostToDevice));
        ng->x.need((size_t)n * c.d_model * 2);
        ng->resid.need((size_t)n * c.d_model * 4);
        // Lane 0 takes half the rows rounded to the 32-row tiles of the linears.
        const int n0 = n_lanes == 1 ? n : std::max(1, ((n / 2 + 16) / 32) * 32);
        ng->n_lanes = n_lanes;
        for (int i = 0; i < n_lanes; ++i) {
            StepLane& ln = ng->lanes[i];
            ln.off = i == 0 ? 0 : n0;
            ln.n = i == 0 ? n0 : n - n0;
            const int r = std::max(ln.n, 1);
            ln.ws.size(c, r);
            ln.ws.part.need(sizeof(float) * decode_part_floats(r, grid) * (c.num_heads / kGroupHeads));
            ln.row_stream.need(sizeof(int32_t) * r);
            ln.row_pos.need(2 * sizeof(int32_t) * r);  // positions, then slots
            ln.prefix.need(sizeof(int32_t) * (r + 1 + kMaxDecodeGrid));
        }
        slot = std::move(ng);
        g = slot.get();
    }
    const int32_t* sid = g->sid.as<int32_t>();
    auto plan_of = [](StepLane& ln) {
        RowPlan plan;
        plan.row_stream = ln.row_stream.as<int32_t>();
        plan.row_pos = ln.row_pos.as<int32_t>();
        plan.row_slot = plan.row_pos + ln.n;
        plan.prefix = ln.prefix.as<int32_t>();
        plan.cta_first = plan.prefix + ln.n + 1;
        return plan;
    };
    inputs(g);
    if (n_lanes > 1 && !model->lane_stream) {
        CK(cudaStreamCreateWithFlags(&model->lane_stream, cudaStreamNonBlocking));
        CK(cudaEventCreateWithFlags(&model->lane_start, cudaEventDisableTiming));
        CK(cudaEventCreateWithFlags(&model->lane_join, cudaEventDisableTiming));
    }
    // `cs2` is the second lane's stream (== cs when the lanes run one after the other).
    auto body = [&](cudaStream_t cs, cudaStream_t cs2, cudaEvent_t* ev) {
        StampLog* stamps = gkey.stamps ? &model->stamps : nullptr;
        if (stamps) {
            CK(cudaMemsetAsync(stamps->buf.p, 0xFF, sizeof(unsigned long long) * 4 * stamps->cap, cs));
            stamps->next = 0;
        }
        if constexpr (!std::is_same_v<std::decay_t<Pre>, std::nullptr_t>) pre(cs);
        for (int i = 0; i < n_lanes; ++i) {
            StepLane& ln = g->lanes[i];
            const cudaStream_t ls = i == 0 ? cs : cs2;
            if (i == 1 && cs2 != cs) CK(cudaStreamWaitEvent(cs2, model->lane_start, 0));
            const RowPlan plan = plan_of(ln);
            launch_plan_decode(kv->len.as<int32_t>(), sid + ln.off, ln.n, kv->streams, kv->capacity, plan,
                               kv->ring(), grid, kv->err.as<uint32_t>(), ls);
            LaneOpts lo;
            lo.id = i;
            lo.lane = n_lanes > 1;
            lo.stamps = stamps;
            lo.after_qkv0 = (i == 0 && n_lanes > 1 && cs2 != cs) ? model->lane_start : nullptr;
            run_layers(model, kv, true, plan, ln.n, g->x.as<__nv_bfloat16>() + (size_t)ln.off * c.d_model,
                       g->resid.as<float>() + (size_t)ln.off * c.d_model, ln.ws, ls,
                       ev ? ev + 2 * c.num_layers * i : nullptr, Tiles{}, lo);
            if constexpr (!std::is_same_v<std::decay_t<Post>, std::nullptr_t>) post(ls, ln.off, ln.n);
        }
        if (n_lanes > 1 && cs2 != cs) {
            CK(cudaEventRecord(model->lane_join, cs2));
            CK(cudaStreamWaitEvent(cs, model->lane_join, 0));
        }
        launch_advance(kv->len.as<int32_t>(), sid, nullptr, n, 1, kv->ring(), kv->capacity, cs);
        check_launch();
    };
    if (tracing_on()) {
        const int L = c.num_layers, E = 2 * L * n_lanes;
        if (model->events.size() < (size_t)(E + 2)) {
            for (cudaEvent_t e : model->events) cudaEventDestroy(e);
            model->events.assign(E + 2, nullptr);
            for (auto& e : model->events) CK(cudaEventCreate(&e));
        }
        cudaEvent_t* ev = model->events.data();
        CK(cudaEventRecord(ev[E], s));
        body(s, s, ev);
        CK(cudaEventRecord(ev[E + 1], s));
        CK(cudaEventSynchronize(ev[E + 1]));
        double bytes = 0.0;  // K and V rows read, f32 q read, bf16 output written
        for (int i = 0; i < n; ++i) bytes += (double)attended_keys(kv, streams_host[i]) * kv->row_bytes * 2;
        bytes += (double)n * kv->heads * kHeadDim * (4 + 2);
        double attn_ms = 0.0;
        for (int l = 0; l < L * n_lanes; ++l) {
            float ms = 0.f;
            CK(cudaEventElapsedTime(&ms, ev[2 * l], ev[2 * l + 1]));
            attn_ms += ms;
        }
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, ev[E], ev[E + 1]));
        trace_add((int64_t)L * n_lanes, attn_ms, bytes * L, 1, ms);
    } else {
        if (!g->exec) {
            cudaStream_t cs = model->capture_stream;
            CK(cudaStreamSynchronize(s));
            CK(cudaStreamBeginCapture(cs, cudaStreamCaptureModeRelaxed));
            try {
                body(cs, n_lanes > 1 ? model->lane_stream : cs, nullptr);
            } catch (...) {
                cudaGraph_t junk = nullptr;
                cudaStreamEndCapture(cs, &junk);
                if (junk) cudaGraphDestroy(junk);
                throw;
            }
            CK(cudaStreamEndCapture(cs, &g->graph));
            CK(cudaGraphInstantiate(&g->exec, g->graph, 0));
        }
        CK(cudaGraphLaunch(g->exec, s));
    }
    for (int i = 0; i < n; ++i) {
        kv->h_len[streams_host[i]] += 1;
        kv->ring_commit(streams_host[i]);
    }
}

// Lets other translation units of the library set this thread's last error.
void ptts_b200_set_last_error(const std::string& msg) { g_last_error = msg; }

extern "C" {

const char* ptts_b200_last_error(void) { return g_last_error.c_str(); }

const char* ptts_b200_version(void) { return "ptts_b200 0.1 sm_100a"; }

int ptts_b200_kv_create(int device, int num_layers, int num_streams, int capacity, int num_heads,
                        int head_dim, int dtype, ptts_b200_kv** out) {
    return guarded([&] {
        require(out != nullptr, PTTS_B200_ERR_ARG, "out is NULL");
        *out = nullptr;
        require(num_layers > 0 && num_streams > 0 && capacity > 0, PTTS_B200_ERR_ARG,
                "layers, streams and capacity must be positive");
        require(head_dim == kHeadDim && num_heads > 0 && num_heads % kGroupHeads == 0, PTTS_B200_ERR_UNSUPPORTED,
                "only head_dim 64 with a multiple of 8 heads is implemented");
        require(dtype == PTTS_B200_F32 || dtype == PTTS_B200_BF16, PTTS_B200_ERR_ARG, "unknown dtype");
        DeviceScope scope(device);
        static uint64_t next_uid = 1;
        auto kv = std::make_unique<ptts_b200_kv>();
        kv->uid = next_uid++;
        kv->device = device;
        kv->layers = num_layers;
        kv->streams = num_streams;
        kv->capacity = capacity;
        kv->heads = num_heads;
        kv->head_dim = head_dim;
        kv->dtype = dtype;
        kv->row_bytes = (size_t)num_heads * head_dim * (dtype == PTTS_B200_BF16 ? 2 : 4);
        const size_t total = (size_t)num_layers * kv->layer_bytes();
        CK(cudaMemset(kv->k.need(total), 0, total));
        CK(cudaMemset(kv->v.need(total), 0, total));
        CK(cudaMemset(kv->len.need(sizeof(int32_t) * num_streams), 0, sizeof(int32_t) * num_streams));
        CK(cudaMemset(kv->err.need(sizeof(uint32_t)), 0, sizeof(uint32_t)));
        kv->h_len.assign(num_streams, 0);
        CK(cudaMemset(kv->ring_write.need(sizeof(int32_t) * num_streams), 0xFF, sizeof(int32_t) * num_streams));
        CK(cudaMemset(kv->ring_filled.need(sizeof(int32_t) * num_streams), 0, sizeof(int32_t) * num_streams));
        CK(cudaMemset(kv->ring_valid.need((size_t)num_streams * capacity), 0, (size_t)num_streams * capacity));
        kv->h_ring_write.assign(num_streams, -1);
        kv->h_ring_filled.assign(num_streams, 0);
        kv->h_ring_valid.assign((size_t)num_streams * capacity, 0);
        CK(cudaMemset(kv->window.need(sizeof(int32_t) * num_streams), 0, sizeof(int32_t) * num_streams));
        kv->h_window.assign(num_streams, 0);
        CK(cudaDeviceSynchronize());
        *out = kv.release();
    });
}

void ptts_b200_kv_destroy(ptts_b200_kv* kv) {
    if (!kv) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(kv->device);
    cudaDeviceSynchronize();
    delete kv;
    if (prev >= 0) cudaSetDevice(prev);
}

int ptts_b200_kv_lengths(const ptts_b200_kv* kv, int32_t* lengths_host) {
    return guarded([&] {
        check_kv(kv);
        require(lengths_host != nullptr, PTTS_B200_ERR_ARG, "lengths_host is NULL");
        std::memcpy(lengths_host, kv->h_len.data(), sizeof(int32_t) * kv->streams);
    });
}

int ptts_b200_kv_pointers(const ptts_b200_kv* kv, int layer, void** k, void** v,
                          int32_t** lengths) {
    return guarded([&] {
        check_kv(kv);
        require(layer >= 0 && layer < kv->layers, PTTS_B200_ERR_ARG, "layer out of range");
        if (k) *k = kv->k_layer(layer);
        if (v) *v = kv->v_layer(layer);
        if (lengths) *lengths = kv->len.as<int32_t>();
    });
}

int ptts_b200_kv_advance(ptts_b200_kv* kv, const int32_t* streams_host, const int32_t* rows_host,
                         int n, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        DeviceScope scope(kv->device);
        std::vector<int32_t> offsets;
        check_sequences(kv, streams_host, rows_host, n, offsets);
        cudaStream_t s = as_stream(cuda_stream);
        std::vector<int32_t> packed(streams_host, streams_host + n);
        packed.insert(packed.end(), offsets.begin(), offsets.end());
        const int32_t* d = kv->upload_seq(packed, s);
        launch_advance(kv->len.as<int32_t>(), d, d + n, n, 0, kv->ring(), kv->capacity, s);
        check_launch();
        for (int i = 0; i < n; ++i) {
            kv->h_len[streams_host[i]] += rows_host[i];
            kv->ring_commit(streams_host[i]);
        }
    });
}

int ptts_b200_kv_reset(ptts_b200_kv* kv, const int32_t* streams_host, int n, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(n > 0 && streams_host, PTTS_B200_ERR_ARG, "no streams");
        for (int i = 0; i < n; ++i)
            require(streams_host[i] >= 0 && streams_host[i] < kv->streams, PTTS_B200_ERR_ARG,
                    "stream out of range");
        DeviceScope scope(kv->device);
        cudaStream_t s = as_stream(cuda_stream);
        const int32_t* d = kv->upload_scratch(streams_host, sizeof(int32_t) * n, s);
        // Every (layer, head group) block in turn: groups() blocks of group_bytes() per layer.
        launch_reset_streams(kv->k.p, kv->v.p, kv->len.as<int32_t>(), d, n, kv->layers * kv->groups(),
                             (long long)kv->group_bytes(), (long long)kv->stream_bytes(), s);
        check_launch();
        for (int i = 0; i < n; ++i) {
            const int st = streams_host[i];
            kv->h_len[st] = 0;
            if (kv->is_ring(st)) ring_clear(kv, st, s);  // back to an appended cache
            if (kv->is_window(st)) {
                kv->h_window[st] = 0;
                kv->staging.upload(kv->window.as<int32_t>() + st, &kv->h_window[st], sizeof(int32_t), s);
            }
        }
    });
}

int ptts_b200_kv_load_prefix(ptts_b200_kv* kv, int layer, int stream, const void* k,
                             const void* v, int len, int set_length, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(layer >= 0 && layer < kv->layers, PTTS_B200_ERR_ARG, "layer out of range");
        require(stream >= 0 && stream < kv->streams, PTTS_B200_ERR_ARG, "stream out of range");
        require(len >= 0, PTTS_B200_ERR_ARG, "negative length");
        require(!kv->is_ring(stream) && !kv->is_window(stream), PTTS_B200_ERR_STATE,
                "a ring or windowed cache cannot load a prefix");
        if (len > kv->capacity)
            fail(PTTS_B200_ERR_CAPACITY, "cannot fit " + std::to_string(len) +
                                             " filled KV positions into a budget of " +
                                             std::to_string(kv->capacity));
        DeviceScope scope(kv->device);
        cudaStream_t s = as_stream(cuda_stream);
        const size_t off = (size_t)stream * kv->stream_bytes();
        if (len > 0) {
            require(k && v, PTTS_B200_ERR_ARG, "k/v are NULL");
            if (kv->groups() == 1) {
                CK(cudaMemcpyAsync(kv->k_layer(layer) + off, k, len * kv->row_bytes, cudaMemcpyDefault, s));
                CK(cudaMemcpyAsync(kv->v_layer(layer) + off, v, len * kv->row_bytes, cudaMemcpyDefault, s));
            } else {
                // [len][H][D] rows into each head group's block: 8 heads of every row per group.
                const size_t gw = kv->group_row_bytes();
                for (int g = 0; g < kv->groups(); ++g) {
                    CK(cudaMemcpy2DAsync(kv->k_group(layer, g) + off, gw, static_cast<const char*>(k) + g * gw,
                                         kv->row_bytes, gw, len, cudaMemcpyDefault, s));
                    CK(cudaMemcpy2DAsync(kv->v_group(layer, g) + off, gw, static_cast<const char*>(v) + g * gw,
                                         kv->row_bytes, gw, len, cudaMemcpyDefault, s));
                }
            }
        }
        if (set_length) {
            kv->h_len[stream] = len;
            kv->staging.upload(kv->len.as<int32_t>() + stream, &len, sizeof(int32_t), s);
        }
    });
}

int ptts_b200_kv_copy_stream(ptts_b200_kv* dst, int dst_stream, const ptts_b200_kv* src,
                             int src_stream, void* cuda_stream) {
    return guarded([&] {
        check_kv(dst);
        check_kv(src);
        require(dst->layers == src->layers && dst->heads == src->heads &&
                    dst->head_dim == src->head_dim && dst->dtype == src->dtype,
                PTTS_B200_ERR_STATE, "the two caches differ in layers, heads or dtype");
        require(dst->device == src->device, PTTS_B200_ERR_STATE, "the two caches are on different devices");
        require(dst_stream >= 0 && dst_stream < dst->streams && src_stream >= 0 &&
                    src_stream < src->streams,
                PTTS_B200_ERR_ARG, "stream out of range");
        require(!src->is_ring(src_stream) && !dst->is_ring(dst_stream), PTTS_B200_ERR_STATE,
                "a ring cache cannot be resized");  // transformer.rs:356-357
        require(!dst->is_window(dst_stream), PTTS_B200_ERR_STATE, "the destination stream is windowed");
        if (src->is_window(src_stream)) {
            // Mimi caches are cloned as they are (transformer.rs:348-355): every slot, the
            // position and the window, so the capacities must match.
            require(dst->capacity == src->capacity, PTTS_B200_ERR_STATE,
                    "a windowed cache is copied whole, into a stream of the same capacity");
            DeviceScope scope(dst->device);
            cudaStream_t s = as_stream(cuda_stream);
            for (int l = 0; l < dst->layers; ++l)
                for (int g = 0; g < dst->groups(); ++g) {
                    CK(cudaMemcpyAsync(dst->k_group(l, g) + (size_t)dst_stream * dst->stream_bytes(),
                                       src->k_group(l, g) + (size_t)src_stream * src->stream_bytes(),
                                       dst->stream_bytes(), cudaMemcpyDeviceToDevice, s));
                    CK(cudaMemcpyAsync(dst->v_group(l, g) + (size_t)dst_stream * dst->stream_bytes(),
                                       src->v_group(l, g) + (size_t)src_stream * src->stream_bytes(),
                                       dst->stream_bytes(), cudaMemcpyDeviceToDevice, s));
                }
            dst->h_len[dst_stream] = src->h_len[src_stream];
            dst->h_window[dst_stream] = src->h_window[src_stream];
            dst->staging.upload(dst->len.as<int32_t>() + dst_stream, &dst->h_len[dst_stream], sizeof(int32_t), s);
            dst->staging.upload(dst->window.as<int32_t>() + dst_stream, &dst->h_window[dst_stream], sizeof(int32_t), s);
            return;
        }
        const int used = src->h_len[src_stream];
        if (used > dst->capacity)
            fail(PTTS_B200_ERR_CAPACITY, "cannot fit " + std::to_string(used) +
                                             " filled KV positions into a budget of " +
                                             std::to_string(dst->capacity));
        DeviceScope scope(dst->device);
        cudaStream_t s = as_stream(cuda_stream);
        for (int lg = 0; lg < dst->layers * dst->groups(); ++lg) {
            const int l = lg / dst->groups(), g = lg % dst->groups();
            char* dk = dst->k_group(l, g) + (size_t)dst_stream * dst->stream_bytes();
            char* dv = dst->v_group(l, g) + (size_t)dst_stream * dst->stream_bytes();
            const char* sk = src->k_group(l, g) + (size_t)src_stream * src->stream_bytes();
            const char* sv = src->v_group(l, g) + (size_t)src_stream * src->stream_bytes();
            const size_t n = (size_t)used * dst->group_row_bytes();
            if (n) {
                CK(cudaMemcpyAsync(dk, sk, n, cudaMemcpyDeviceToDevice, s));
                CK(cudaMemcpyAsync(dv, sv, n, cudaMemcpyDeviceToDevice, s));
            }
            CK(cudaMemsetAsync(dk + n, 0, dst->stream_bytes() - n, s));
            CK(cudaMemsetAsync(dv + n, 0, dst->stream_bytes() - n, s));
        }
        dst->h_len[dst_stream] = used;
        dst->staging.upload(dst->len.as<int32_t>() + dst_stream, &used, sizeof(int32_t), s);
    });
}

int ptts_b200_kv_check(ptts_b200_kv* kv) {
    return guarded([&] {
        check_kv(kv);
        DeviceScope scope(kv->device);
        CK(cudaDeviceSynchronize());
        uint32_t e = 0;
        CK(cudaMemcpy(&e, kv->err.p, sizeof(e), cudaMemcpyDeviceToHost));
        CK(cudaMemset(kv->err.p, 0, sizeof(e)));
        if (e) {
            std::string what;
            if (e & DEV_ERR_BOUNDS) what += " bounds";
            if (e & DEV_ERR_CAPACITY) what += " capacity";
            if (e & DEV_ERR_TIMEOUT) what += " timeout";
            if (e & DEV_ERR_DUPLICATE) what += " duplicate";
            fail(PTTS_B200_ERR_DEVICE, "device-side check tripped:" + what);
        }
    });
}

int ptts_b200_attend(ptts_b200_kv* kv, int layer, const void* q, const void* k, const void* v,
                     int in_dtype, int num_kv_heads, const int32_t* streams_host,
                     const int32_t* rows_host, int n_seq, float max_period, void* out,
                     int out_dtype, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(layer >= 0 && layer < kv->layers, PTTS_B200_ERR_ARG, "layer out of range");
        require(q && k && v && out, PTTS_B200_ERR_ARG, "q/k/v/out are NULL");
        require(in_dtype == PTTS_B200_F32 || in_dtype == PTTS_B200_BF16, PTTS_B200_ERR_ARG, "bad in_dtype");
        require(out_dtype == PTTS_B200_F32 || out_dtype == PTTS_B200_BF16, PTTS_B200_ERR_ARG, "bad out_dtype");
        require(num_kv_heads > 0 && kv->heads % num_kv_heads == 0, PTTS_B200_ERR_ARG,
                "the " + std::to_string(num_kv_heads) + " key/value heads do not divide the " +
                    std::to_string(kv->heads) + " attention heads");
        require(max_period > 1.0f, PTTS_B200_ERR_ARG, "max_period must be above 1");
        std::vector<int32_t> offsets;
        const int n_rows = check_sequences(kv, streams_host, rows_host, n_seq, offsets);
        bool decode = true;
        for (int i = 0; i < n_seq; ++i) decode = decode && rows_host[i] == 1;
        refuse_ring_prompt(kv, streams_host, n_seq, decode);
        DeviceScope scope(kv->device);
        cudaStream_t s = as_stream(cuda_stream);
        std::vector<int32_t> packed(streams_host, streams_host + n_seq);
        packed.insert(packed.end(), offsets.begin(), offsets.end());
        // A prompt's tile list travels in the same copy (8-byte aligned after the lists).
        const std::vector<int2> tl = decode ? std::vector<int2>{} : make_tiles(offsets, streams_host, kv->h_len);
        const size_t tile_at = append_tiles(packed, tl);
        const int32_t* d = kv->upload_seq(packed, s);
        const RowPlan plan = make_plan(kv, decode, d, d + n_seq, n_seq, n_rows, kv->row_stream,
                                       kv->row_pos, kv->prefix, s);
        check_launch();
        RopeAppendArgs ra{};
        ra.q = q;
        ra.k = k;
        ra.v = v;
        const size_t hd = (size_t)kv->heads * kHeadDim;
        ra.q_out = static_cast<float*>(kv->q_rot.need((size_t)n_rows * hd * sizeof(float)));
        ra.k_cache = kv->k_layer(layer);
        ra.v_cache = kv->v_layer(layer);
        ra.row_stream = plan.row_stream;
        ra.row_pos = plan.row_pos;
        ra.row_slot = plan.row_slot;
        ra.rows = n_rows;
        ra.heads = kv->heads;
        ra.kv_heads = num_kv_heads;
        ra.num_streams = kv->streams;
        ra.capacity = kv->capacity;
        rope_inv_freq(kv->head_dim, max_period, ra.inv_freq);
        ra.err = kv->err.as<uint32_t>();
        bool windowed = false;
        for (int i = 0; i < n_seq; ++i) windowed = windowed || kv->is_window(streams_host[i]);
        if (prefill_fa(kv->dtype == PTTS_B200_BF16, decode, windowed)) {
            ra.q_hi = reinterpret_cast<__nv_bfloat16*>(ra.q_out);  // two bf16 planes in the f32 buffer
            ra.q_lo = ra.q_hi + (size_t)n_rows * hd;
            ra.q_scale = (1.0f / sqrtf((float)kv->head_dim)) * kLog2e;  // transformer.rs:215, exp2 domain
        }
        launch_rope_append(ra, in_dtype == PTTS_B200_BF16, kv->dtype == PTTS_B200_BF16, s);
        check_launch();
        const bool trace = decode && tracing_on();
        if (trace) {
            for (auto& e : kv->trace_ev)
                if (!e) CK(cudaEventCreate(&e));
            CK(cudaEventRecord(kv->trace_ev[0], s));
        }
        Tiles tiles;
        if (!decode) {
            tiles.dev = reinterpret_cast<const int2*>(d + tile_at);
            tiles.n = (int)tl.size();
            tiles.windowed = windowed;
        }
        attention(kv, layer, decode, plan, n_rows, ra.q_out, out, nullptr,
                  out_dtype == PTTS_B200_BF16 ? kOutBf16 : kOutF32, kv->part, kv->counters, tiles, s);
        if (trace) {
            CK(cudaEventRecord(kv->trace_ev[1], s));
            CK(cudaEventSynchronize(kv->trace_ev[1]));
            float ms = 0.f;
            CK(cudaEventElapsedTime(&ms, kv->trace_ev[0], kv->trace_ev[1]));
            double bytes = 0.0;
            for (int i = 0; i < n_seq; ++i)
                bytes += (double)attended_keys(kv, streams_host[i]) * kv->row_bytes * 2;
            bytes += (double)n_seq * hd * (4 + (out_dtype == PTTS_B200_BF16 ? 2 : 4));
            trace_add(1, ms, bytes, 0, 0.0);
        }
    });
}

int ptts_b200_linear_i8(int device, const void* x, const int8_t* w, const float* scale, int m,
                        int n, int k, float* y, void* cuda_stream) {
    return guarded([&] {
        require(x && w && scale && y, PTTS_B200_ERR_ARG, "NULL argument");
        require(m > 0 && n > 0 && k > 0, PTTS_B200_ERR_ARG, "sizes must be positive");
        require(n % 64 == 0 && k % 64 == 0, PTTS_B200_ERR_UNSUPPORTED, "n and k must be multiples of 64");
        DeviceScope scope(device);
        LinearArgs a{};
        a.M = m;
        a.N = n;
        a.K = k;
        a.a = x;
        a.a_f16 = 0;  // one bf16 plane
        a.w = w;
        a.scale = scale;
        a.y = y;
        require(launch_linear(a, EPI_F32, as_stream(cuda_stream)), PTTS_B200_ERR_UNSUPPORTED,
                "no kernel for this linear's shape");
        check_launch();
    });
}

int ptts_b200_model_create(int device, const ptts_b200_config* config, ptts_b200_model** out) {
    return guarded([&] {
        require(out && config, PTTS_B200_ERR_ARG, "NULL argument");
        *out = nullptr;
        const ptts_b200_config& c = *config;
        // transformer.rs:699-707
        if (c.num_heads <= 0 || c.num_heads * c.head_dim <= 0)
            fail(PTTS_B200_ERR_ARG, "the config's " + std::to_string(c.num_heads) +
                                        " attention heads do not divide its width");
        if (c.num_kv_heads <= 0 || c.num_heads % c.num_kv_heads != 0)
            fail(PTTS_B200_ERR_ARG, "the config's " + std::to_string(c.num_kv_heads) +
                                        " key/value heads do not divide its " +
                                        std::to_string(c.num_heads) + " attention heads");
        require(c.head_dim == kHeadDim && c.num_heads % kGroupHeads == 0, PTTS_B200_ERR_UNSUPPORTED,
                "only head_dim 64 with a multiple of 8 heads is implemented");
        require(c.d_model > 0 && c.d_model % 128 == 0 && c.d_model <= 1024, PTTS_B200_ERR_UNSUPPORTED,
                "d_model must be a multiple of 128 up to 1024");
        require(c.dim_feedforward > 0 && c.dim_feedforward % 64 == 0, PTTS_B200_ERR_UNSUPPORTED,
                "dim_feedforward must be a multiple of 64");
        require(c.num_layers > 0, PTTS_B200_ERR_ARG, "num_layers must be positive");
        require(c.max_period > 1.0f, PTTS_B200_ERR_ARG, "max_period must be above 1");
        require(c.gelu == 0 || c.gelu == 1, PTTS_B200_ERR_ARG, "gelu is 0 (erf) or 1 (tanh)");
        DeviceScope scope(device);
        auto m = std::make_unique<ptts_b200_model>();
        m->device = device;
        m->cfg = c;
        rope_inv_freq(c.head_dim, c.max_period, m->inv_freq);
        for (int l = 0; l < c.num_layers; ++l) m->layers.push_back(std::make_unique<ptts_b200_model::Layer>());
        CK(cudaStreamCreateWithFlags(&m->capture_stream, cudaStreamNonBlocking));
        *out = m.release();
    });
}

void ptts_b200_model_destroy(ptts_b200_model* model) {
    if (!model) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(model->device);
    cudaDeviceSynchronize();
    delete model;
    if (prev >= 0) cudaSetDevice(prev);
}

int ptts_b200_model_load_layer(ptts_b200_model* model, int layer,
                               const ptts_b200_layer_weights* w) {
    return guarded([&] {
        require(model && w, PTTS_B200_ERR_ARG, "NULL argument");
        require(layer >= 0 && layer < model->cfg.num_layers, PTTS_B200_ERR_ARG, "layer out of range");
        const ptts_b200_config& c = model->cfg;
        const size_t dm = c.d_model, hd = (size_t)c.num_heads * c.head_dim;
        const size_t nqkv = hd + 2 * (size_t)c.num_kv_heads * c.head_dim, ff = c.dim_feedforward;
        require(w->in_proj_host && w->in_proj_scale_host && w->out_proj_host &&
                    w->out_proj_scale_host && w->linear1_host && w->linear1_scale_host &&
                    w->linear2_host && w->linear2_scale_host && w->norm1_weight_host &&
                    w->norm1_bias_host && w->norm2_weight_host && w->norm2_bias_host,
                PTTS_B200_ERR_ARG, "a weight pointer is NULL");
        DeviceScope scope(model->device);
        auto& L = *model->layers[layer];
        auto put = [](DevBuf& b, const void* src, size_t n) {
            CK(cudaMemcpy(b.need(n), src, n, cudaMemcpyHostToDevice));
        };
        put(L.w_qkv, w->in_proj_host, nqkv * dm);
        put(L.s_qkv, w->in_proj_scale_host, nqkv * 4);
        put(L.w_out, w->out_proj_host, dm * hd);
        put(L.s_out, w->out_proj_scale_host, dm * 4);
        const float* so = static_cast<const float*>(w->out_proj_scale_host);
        L.base_out.assign(so, so + dm);
        put(L.w1, w->linear1_host, ff * dm);
        put(L.s1, w->linear1_scale_host, ff * 4);
        put(L.w2, w->linear2_host, dm * ff);
        put(L.s2, w->linear2_scale_host, dm * 4);
        const float* s2 = static_cast<const float*>(w->linear2_scale_host);
        L.base_2.assign(s2, s2 + dm);
        apply_layer_scale(L);
        put(L.ln1g, w->norm1_weight_host, dm * 4);
        put(L.ln1b, w->norm1_bias_host, dm * 4);
        put(L.ln2g, w->norm2_weight_host, dm * 4);
        put(L.ln2b, w->norm2_bias_host, dm * 4);
        for (DevBuf* b : {&L.l_qkv, &L.l_out, &L.l1, &L.l2}) b->release();  // int8 layers: one plane
        // The tcgen05 linears read the int8 weights and widen them on chip. An exact f16 copy of
        // every weight, read instead (twice the bytes), is kept only with PTTS_B200_WEIGHTS=f16.
        const char* wsel = getenv("PTTS_B200_WEIGHTS");
        if (wsel && wsel[0] == 'f') {
            auto widen = [](DevBuf& h, const DevBuf& q, size_t n) {
                launch_i8_to_f16(q.as<int8_t>(), static_cast<__half*>(h.need(n * 2)), (long long)n, nullptr);
            };
            widen(L.h_qkv, L.w_qkv, nqkv * dm);
            widen(L.h_out, L.w_out, dm * hd);
            widen(L.h1, L.w1, ff * dm);
            widen(L.h2, L.w2, dm * ff);
        } else {
            for (DevBuf* b : {&L.h_qkv, &L.h_out, &L.h1, &L.h2}) b->release();
        }
        check_launch();
        CK(cudaDeviceSynchronize());
        L.loaded = true;
    });
}

int ptts_b200_model_set_layer_scale(ptts_b200_model* model, int layer, const float* scale1_host,
                                    const float* scale2_host) {
    return guarded([&] {
        require(model != nullptr, PTTS_B200_ERR_ARG, "model is NULL");
        require(layer >= 0 && layer < model->cfg.num_layers, PTTS_B200_ERR_ARG, "layer out of range");
        const size_t dm = model->cfg.d_model;
        auto take = [&](const float* src, std::vector<float>& dst) {
            if (!src) {
                dst.clear();
                return;
            }
            for (size_t i = 0; i < dm; ++i) require(std::isfinite(src[i]), PTTS_B200_ERR_ARG, "a layer scale is not finite");
            dst.assign(src, src + dm);
        };
        DeviceScope scope(model->device);
        auto& L = *model->layers[layer];
        take(scale1_host, L.ls1);
        take(scale2_host, L.ls2);
        apply_layer_scale(L);
        CK(cudaDeviceSynchronize());
    });
}

int ptts_b200_model_config(const ptts_b200_model* model, ptts_b200_config* out) {
    return guarded([&] {
        require(model && out, PTTS_B200_ERR_ARG, "NULL argument");
        *out = model->cfg;
    });
}

int ptts_b200_model_load_layer_f32(ptts_b200_model* model, int layer, const ptts_b200_layer_weights_f32* w) {
    return guarded([&] {
        require(model && w, PTTS_B200_ERR_ARG, "NULL argument");
        load_dense_layer(model, layer, w->in_proj_host, w->out_proj_host, w->linear1_host, w->linear2_host,
                         w->norm1_weight_host, w->norm1_bias_host, w->norm2_weight_host, w->norm2_bias_host);
    });
}

int ptts_b200_model_load_layer_q8_0(ptts_b200_model* model, int layer, const ptts_b200_layer_weights_q8_0* w) {
    return guarded([&] {
        require(model && w, PTTS_B200_ERR_ARG, "NULL argument");
        require(w->in_proj_q8_0 && w->out_proj_q8_0 && w->linear1_q8_0 && w->linear2_q8_0, PTTS_B200_ERR_ARG,
                "a weight pointer is NULL");
        const ptts_b200_config& c = model->cfg;
        const size_t dm = c.d_model, hd = (size_t)c.num_heads * c.head_dim;
        const size_t nqkv = hd + 2 * (size_t)c.num_kv_heads * c.head_dim, ff = c.dim_feedforward;
        require(dm % 32 == 0 && hd % 32 == 0 && ff % 32 == 0, PTTS_B200_ERR_UNSUPPORTED,
                "q8_0 needs every input width to be a multiple of 32");
        const auto qkv = dequant_q8_0(w->in_proj_q8_0, nqkv, dm), out = dequant_q8_0(w->out_proj_q8_0, dm, hd);
        const auto l1 = dequant_q8_0(w->linear1_q8_0, ff, dm), l2 = dequant_q8_0(w->linear2_q8_0, dm, ff);
        load_dense_layer(model, layer, qkv.data(), out.data(), l1.data(), l2.data(), w->norm1_weight_host,
                         w->norm1_bias_host, w->norm2_weight_host, w->norm2_bias_host);
        DeviceScope scope(model->device);
        auto& L = *model->layers[layer];
        // All four linears in the on-chip form, or none (the layer then reads its planes).
        const bool all = upload_q8_blocks(L.q8_qkv, L.bq_qkv, w->in_proj_q8_0, qkv.data(), nqkv, dm) &&
                         upload_q8_blocks(L.q8_out, L.bq_out, w->out_proj_q8_0, out.data(), dm, hd) &&
                         upload_q8_blocks(L.q8_1, L.bq1, w->linear1_q8_0, l1.data(), ff, dm) &&
                         upload_q8_blocks(L.q8_2, L.bq2, w->linear2_q8_0, l2.data(), dm, ff);
        if (!all)
            for (DevBuf* b : {&L.q8_qkv, &L.q8_out, &L.q8_1, &L.q8_2, &L.bq_qkv, &L.bq_out, &L.bq1, &L.bq2})
                b->release();
    });
}

int ptts_b200_forward(ptts_b200_model* model, ptts_b200_kv* kv, const void* x,
                      const int32_t* streams_host, const int32_t* rows_host, int n_seq, float* y,
                      void* cuda_stream) {
    return guarded([&] {
        check_model_kv(model, kv);
        require(x && y, PTTS_B200_ERR_ARG, "x/y are NULL");
        std::vector<int32_t> offsets;
        const int rows = check_sequences(kv, streams_host, rows_host, n_seq, offsets);
        bool decode = true;
        for (int i = 0; i < n_seq; ++i) decode = decode && rows_host[i] == 1;
        refuse_ring_prompt(kv, streams_host, n_seq, decode);
        DeviceScope scope(model->device);
        cudaStream_t s = as_stream(cuda_stream);
        const ptts_b200_config& c = model->cfg;
        // RoPE factors for every position of the call: a windowed stream's (Mimi's
        // absolute_offset) grows past the capacity.
        long long rope_need = kv->capacity;
        bool windowed = false;
        for (int i = 0; i < n_seq; ++i)
            if (kv->is_window(streams_host[i])) {
                windowed = true;
                rope_need = std::max<long long>(rope_need, (long long)kv->h_len[streams_host[i]] + rows_host[i]);
            }
        ensure_rope(model, (int)rope_need, s);
        std::vector<int32_t> packed(streams_host, streams_host + n_seq);
        packed.insert(packed.end(), offsets.begin(), offsets.end());
        // A prompt's tile list travels in the same copy.
        const std::vector<int2> tl = decode ? std::vector<int2>{} : make_tiles(offsets, streams_host, kv->h_len);
        const size_t tile_at = append_tiles(packed, tl);
        int32_t* d = static_cast<int32_t*>(model->seq_stream.need(sizeof(int32_t) * packed.size()));
        model->staging.upload(d, packed.data(), sizeof(int32_t) * packed.size(), s);
        const RowPlan plan = make_plan(kv, decode, d, d + n_seq, n_seq, rows, model->row_stream,
                                       model->row_pos, model->prefix, s);
        check_launch();
        model->ws.size(c, rows);
        Tiles tiles;
        if (!decode) {
            tiles.dev = reinterpret_cast<const int2*>(d + tile_at);
            tiles.n = (int)tl.size();
            tiles.windowed = windowed;
        }
        // The residual stream lives in the caller's output y.
        run_layers(model, kv, decode, plan, rows, static_cast<const __nv_bfloat16*>(x), y, model->ws, s,
                   nullptr, tiles);
        launch_advance(kv->len.as<int32_t>(), d, d + n_seq, n_seq, 0, kv->ring(), kv->capacity, s);
        check_launch();
        for (int i = 0; i < n_seq; ++i) {
            kv->h_len[streams_host[i]] += rows_host[i];
            kv->ring_commit(streams_host[i]);
        }
    });
}

int ptts_b200_step(ptts_b200_model* model, ptts_b200_kv* kv, const int32_t* streams_host, int n,
                   const void* x, float* y, void* cuda_stream) {
    return guarded([&] {
        check_model_kv(model, kv);
        require(x && y, PTTS_B200_ERR_ARG, "x/y are NULL");
        DeviceScope scope(model->device);
        cudaStream_t s = as_stream(cuda_stream);
        const ptts_b200_config& c = model->cfg;
        const size_t xb = (size_t)n * c.d_model * 2, yb = (size_t)n * c.d_model * 4;
        StepGraph* g = nullptr;
        run_step(model, kv, streams_host, n, model->step, GraphKey{}, s,
                 [&](StepGraph* sg) {
                     g = sg;
                     CK(cudaMemcpyAsync(g->x.p, x, xb,
                                        is_device_pointer(x) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s));
                 },
                 nullptr, nullptr);
        CK(cudaMemcpyAsync(y, g->resid.p, yb, is_device_pointer(y) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, s));
    });
}

int ptts_b200_frame(ptts_b200_model* model, ptts_b200_flow* flow, ptts_b200_kv* kv, const int32_t* streams_host,
                    int n, const float* latent_in, const float* noise, float* latent_out, float* eos,
                    void* cuda_stream) {
    return guarded([&] {
        check_model_kv(model, kv);
        require(flow && noise && latent_out && eos, PTTS_B200_ERR_ARG, "NULL argument");
        DeviceScope scope(model->device);
        cudaStream_t s = as_stream(cuda_stream);
        const uint64_t version = ptts_b200_flow_prepare(flow, n > 0 ? n : 1, model->cfg.d_model);
        const size_t lb = (size_t)n * ptts_b200_flow_ldim(flow) * 4;
        const bool bos = latent_in == nullptr;
        GraphKey key;
        key.flow = version;
        key.bos = bos;
        auto kind = [](const void* p) {
            return is_device_pointer(p) ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
        };
        StepGraph* g = nullptr;
        run_step(model, kv, streams_host, n, model->frame, key, s,
                 [&](StepGraph* sg) {  // inputs into the graph's own buffers
                     g = sg;
                     g->lat_in.need(lb);
                     g->noise.need(lb);
                     g->lat_out.need(lb);
                     g->eos.need((size_t)n * 4);
                     if (!bos) CK(cudaMemcpyAsync(g->lat_in.p, latent_in, lb, kind(latent_in), s));
                     CK(cudaMemcpyAsync(g->noise.p, noise, lb, kind(noise), s));
                 },
                 [&](cudaStream_t cs) {  // input_linear, inside the recorded body
                     ptts_b200_flow_input(flow, bos ? nullptr : g->lat_in.as<float>(), g->x.as<__nv_bfloat16>(), n, cs);
                 },
                 [&](cudaStream_t cs, int off, int rows) {  // out_norm, EOS and the flow net, per lane
                     const int ld = ptts_b200_flow_ldim(flow);
                     ptts_b200_flow_head(flow, g->resid.as<float>() + (size_t)off * model->cfg.d_model, rows,
                                         g->noise.as<float>() + (size_t)off * ld,
                                         g->lat_out.as<float>() + (size_t)off * ld, g->eos.as<float>() + off, cs, off);
                 });
        auto back = [](const void* p) {
            return is_device_pointer(p) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
        };
        CK(cudaMemcpyAsync(latent_out, g->lat_out.p, lb, back(latent_out), s));
        CK(cudaMemcpyAsync(eos, g->eos.p, (size_t)n * 4, back(eos), s));
    });
}

int ptts_b200_model_stamps(ptts_b200_model* model, int max_launches) {
    return guarded([&] {
        require(model != nullptr, PTTS_B200_ERR_ARG, "model is NULL");
        require(max_launches >= 0, PTTS_B200_ERR_ARG, "max_launches must be >= 0");
        DeviceScope scope(model->device);
        CK(cudaDeviceSynchronize());
        StampLog& st = model->stamps;
        if (max_launches > 0) st.buf.need(sizeof(unsigned long long) * 4 * (size_t)max_launches);
        st.cap = max_launches;
        st.next = 0;
        st.meta.assign((size_t)max_launches, ptts_b200_stamp{});
    });
}

int ptts_b200_model_stamps_read(ptts_b200_model* model, ptts_b200_stamp* out, int max, int* n) {
    return guarded([&] {
        require(model != nullptr && out != nullptr && n != nullptr, PTTS_B200_ERR_ARG, "NULL argument");
        DeviceScope scope(model->device);
        const StampLog& st = model->stamps;
        require(st.cap > 0, PTTS_B200_ERR_STATE, "stamps are off (ptts_b200_model_stamps)");
        CK(cudaDeviceSynchronize());
        std::vector<unsigned long long> w((size_t)4 * st.next);
        if (st.next > 0) CK(cudaMemcpy(w.data(), st.buf.p, w.size() * 8, cudaMemcpyDeviceToHost));
        unsigned long long t0 = ~0ull;
        for (int i = 0; i < st.next; ++i) t0 = std::min(t0, w[4 * i + STAMP_ENTRY]);
        auto us = [&](unsigned long long t) { return t == ~0ull ? -1.0 : (double)(t - t0) / 1000.0; };
        const int k = std::min(max, st.next);
        for (int i = 0; i < k; ++i) {
            out[i] = st.meta[i];
            out[i].entry_us = us(w[4 * i + STAMP_ENTRY]);
            out[i].start_us = us(w[4 * i + STAMP_START]);
            const unsigned long long e = w[4 * i + STAMP_END], le = w[4 * i + STAMP_LAST_ENTRY];
            out[i].end_us = e == ~0ull ? -1.0 : us(~e);
            out[i].last_entry_us = le == ~0ull ? -1.0 : us(~le);
        }
        *n = k;
    });
}

int ptts_b200_set_tracing(int on) {
    return guarded([&] {
        std::lock_guard<std::mutex> g(tracer().mu);
        tracer().on = on != 0;
    });
}

int ptts_b200_trace_read(ptts_b200_trace* out, int reset) {
    return guarded([&] {
        require(out != nullptr, PTTS_B200_ERR_ARG, "out is NULL");
        std::lock_guard<std::mutex> g(tracer().mu);
        *out = tracer().t;
        if (reset) tracer().t = ptts_b200_trace{};
    });
}

int ptts_b200_kv_start_ring(ptts_b200_kv* kv, const int32_t* streams_host, int n, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(n > 0 && streams_host, PTTS_B200_ERR_ARG, "no streams");
        for (int i = 0; i < n; ++i) {
            const int st = streams_host[i];
            require(st >= 0 && st < kv->streams, PTTS_B200_ERR_ARG, "stream out of range");
            if (kv->is_ring(st)) fail(PTTS_B200_ERR_STATE, "stream " + std::to_string(st) + " is already a ring");
            if (kv->is_window(st)) fail(PTTS_B200_ERR_STATE, "stream " + std::to_string(st) + " is windowed");
        }
        DeviceScope scope(kv->device);
        cudaStream_t s = as_stream(cuda_stream);
        for (int i = 0; i < n; ++i) {
            // start_ring (transformer.rs:842-852): the rows so far stay, the next goes after them.
            const int st = streams_host[i], used = kv->h_len[st];
            kv->h_ring_write[st] = used;
            kv->h_ring_filled[st] = used;
            uint8_t* hv = kv->h_ring_valid.data() + (size_t)st * kv->capacity;
            std::fill(hv, hv + kv->capacity, 0);
            std::fill(hv, hv + used, 1);
            kv->staging.upload(kv->ring_write.as<int32_t>() + st, &kv->h_ring_write[st], sizeof(int32_t), s);
            kv->staging.upload(kv->ring_filled.as<int32_t>() + st, &kv->h_ring_filled[st], sizeof(int32_t), s);
            uint8_t* dv = kv->ring_valid.as<uint8_t>() + (size_t)st * kv->capacity;
            if (used > 0) CK(cudaMemsetAsync(dv, 1, used, s));
            if (used < kv->capacity) CK(cudaMemsetAsync(dv + used, 0, kv->capacity - used, s));
        }
    });
}

int ptts_b200_kv_set_window(ptts_b200_kv* kv, const int32_t* streams_host, int n, int context,
                            void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(n > 0 && streams_host, PTTS_B200_ERR_ARG, "no streams");
        require(context >= 1 && context <= kv->capacity, PTTS_B200_ERR_ARG,
                "context must be in 1.." + std::to_string(kv->capacity) + " (the capacity)");
        for (int i = 0; i < n; ++i) {
            const int st = streams_host[i];
            require(st >= 0 && st < kv->streams, PTTS_B200_ERR_ARG, "stream out of range");
            if (kv->is_ring(st)) fail(PTTS_B200_ERR_STATE, "stream " + std::to_string(st) + " is a ring");
            if (kv->h_len[st] != 0)
                fail(PTTS_B200_ERR_STATE, "stream " + std::to_string(st) + " is not empty (KvCache::new starts a window)");
        }
        DeviceScope scope(kv->device);
        cudaStream_t s = as_stream(cuda_stream);
        for (int i = 0; i < n; ++i) {
            kv->h_window[streams_host[i]] = context;
            kv->staging.upload(kv->window.as<int32_t>() + streams_host[i], &context, sizeof(int32_t), s);
        }
    });
}

int ptts_b200_kv_set_ring_slot(ptts_b200_kv* kv, int stream, int slot, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(stream >= 0 && stream < kv->streams, PTTS_B200_ERR_ARG, "stream out of range");
        require(kv->is_ring(stream), PTTS_B200_ERR_STATE, "not a ring cache, see ptts_b200_kv_start_ring");
        require(slot >= 0 && slot < kv->capacity, PTTS_B200_ERR_ARG,
                "slot " + std::to_string(slot) + " of a " + std::to_string(kv->capacity) + "-slot ring");
        DeviceScope scope(kv->device);
        kv->h_ring_write[stream] = slot;
        kv->staging.upload(kv->ring_write.as<int32_t>() + stream, &kv->h_ring_write[stream], sizeof(int32_t),
                           as_stream(cuda_stream));
    });
}

int ptts_b200_kv_set_ring_slots(ptts_b200_kv* kv, const int32_t* streams_host, const int32_t* slots_host,
                                int n, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(n > 0 && streams_host && slots_host, PTTS_B200_ERR_ARG, "no streams");
        std::vector<char> seen(kv->streams, 0);
        for (int i = 0; i < n; ++i) {
            const int st = streams_host[i], slot = slots_host[i];
            require(st >= 0 && st < kv->streams, PTTS_B200_ERR_ARG, "stream out of range");
            require(!seen[st], PTTS_B200_ERR_ARG, "stream " + std::to_string(st) + " appears twice");
            seen[st] = 1;
            require(kv->is_ring(st), PTTS_B200_ERR_STATE, "not a ring cache, see ptts_b200_kv_start_ring");
            require(slot >= 0 && slot < kv->capacity, PTTS_B200_ERR_ARG,
                    "slot " + std::to_string(slot) + " of a " + std::to_string(kv->capacity) + "-slot ring");
        }
        DeviceScope scope(kv->device);
        cudaStream_t s = as_stream(cuda_stream);
        // The same int32 scatter as set_lengths, into the write slots.
        if (n <= kSetLengthsInline) {
            SetLengthsInline l;
            l.n = n;
            std::memcpy(l.stream, streams_host, sizeof(int32_t) * n);
            std::memcpy(l.value, slots_host, sizeof(int32_t) * n);
            launch_set_lengths_inline(kv->ring_write.as<int32_t>(), l, s);
        } else {
            std::vector<int32_t> packed(streams_host, streams_host + n);
            packed.insert(packed.end(), slots_host, slots_host + n);
            const int32_t* d = kv->upload_scratch(packed.data(), sizeof(int32_t) * packed.size(), s);
            launch_set_lengths(kv->ring_write.as<int32_t>(), d, d + n, n, s);
        }
        check_launch();
        for (int i = 0; i < n; ++i) kv->h_ring_write[streams_host[i]] = slots_host[i];
    });
}

int ptts_b200_kv_evict(ptts_b200_kv* kv, int stream, int prefix, const int32_t* slots_host, int n,
                       float max_period, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(stream >= 0 && stream < kv->streams, PTTS_B200_ERR_ARG, "stream out of range");
        require(kv->is_ring(stream), PTTS_B200_ERR_STATE, "not a ring cache, see ptts_b200_kv_start_ring");
        require(n >= 0 && (n == 0 || slots_host), PTTS_B200_ERR_ARG, "slots are NULL");
        require(prefix >= 0, PTTS_B200_ERR_ARG, "negative prefix");
        require(max_period > 1.0f, PTTS_B200_ERR_ARG, "max_period must be above 1");
        require(n <= kv->h_len[stream], PTTS_B200_ERR_ARG,
                "cannot evict " + std::to_string(n) + " of " + std::to_string(kv->h_len[stream]) + " positions");
        // Every slot is checked before anything changes, so a refused call leaves the cache as is.
        uint8_t* hv = kv->h_ring_valid.data() + (size_t)stream * kv->capacity;
        std::vector<char> seen(kv->capacity, 0);
        for (int i = 0; i < n; ++i) {
            const int sl = slots_host[i];
            if (sl < prefix || sl >= kv->capacity || !hv[sl] || seen[sl])
                fail(PTTS_B200_ERR_ARG, "slot " + std::to_string(sl) + " holds no row past the prefix");
            seen[sl] = 1;
        }
        if (n == 0) return;
        DeviceScope scope(kv->device);
        cudaStream_t s = as_stream(cuda_stream);
        RingEvictArgs a{};
        const int32_t* d = kv->upload_scratch(slots_host, sizeof(int32_t) * n, s);
        a.k_cache = kv->k.p;
        a.layers = kv->layers;
        const long long elem = kv->dtype == PTTS_B200_BF16 ? 2 : 4;
        a.layer_elems = (long long)kv->layer_bytes() / elem;
        a.streams = kv->streams;
        a.row_elems = kv->heads * kv->head_dim;
        a.capacity = kv->capacity;
        a.sid = stream;
        a.prefix = prefix;
        a.filled = kv->h_ring_filled[stream];
        a.shift = n;
        a.bf16 = kv->dtype == PTTS_B200_BF16;
        rope_inv_freq(kv->head_dim, max_period, a.inv_freq);
        a.slots = d;
        a.n = n;
        a.ring = kv->ring();
        a.lengths = kv->len.as<int32_t>();
        launch_ring_evict(a, s);
        check_launch();
        for (int i = 0; i < n; ++i) hv[slots_host[i]] = 0;
        kv->h_len[stream] -= n;
    });
}

int ptts_b200_kv_set_lengths(ptts_b200_kv* kv, const int32_t* streams_host,
                             const int32_t* lengths_host, int n, void* cuda_stream) {
    return guarded([&] {
        check_kv(kv);
        require(n > 0 && streams_host && lengths_host, PTTS_B200_ERR_ARG, "no streams");
        for (int i = 0; i < n; ++i) {
            require(streams_host[i] >= 0 && streams_host[i] < kv->streams, PTTS_B200_ERR_ARG,
                    "stream out of range");
            require(!kv->is_ring(streams_host[i]), PTTS_B200_ERR_STATE,
                    "a ring cache drops rows by eviction (ptts_b200_kv_evict), not by length");
            require(!kv->is_window(streams_host[i]), PTTS_B200_ERR_STATE,
                    "a windowed cache keeps its position; reset it to start over");
            if (lengths_host[i] < 0 || lengths_host[i] > kv->capacity)
                fail(PTTS_B200_ERR_CAPACITY, "cannot fit " + std::to_string(lengths_host[i]) +
                                                 " filled KV positions into a budget of " +
                                                 std::to_string(kv->capacity));
        }
        DeviceScope scope(kv->device);
        cudaStream_t s = as_stream(cuda_stream);
        if (n <= kSetLengthsInline) {  // a short list rides in the launch, no copy
            SetLengthsInline l;
            l.n = n;
            std::memcpy(l.stream, streams_host, sizeof(int32_t) * n);
            std::memcpy(l.value, lengths_host, sizeof(int32_t) * n);
            launch_set_lengths_inline(kv->len.as<int32_t>(), l, s);
        } else {
            std::vector<int32_t> packed(streams_host, streams_host + n);
            packed.insert(packed.end(), lengths_host, lengths_host + n);
            const int32_t* d = kv->upload_scratch(packed.data(), sizeof(int32_t) * packed.size(), s);
            launch_set_lengths(kv->len.as<int32_t>(), d, d + n, n, s);
        }
        check_launch();
        for (int i = 0; i < n; ++i) kv->h_len[streams_host[i]] = lengths_host[i];
    });
}

}  // extern "C"
