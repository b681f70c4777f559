// Decode attention that allocates nothing: ptts_b200_attend_decode_noalloc.
//
// Who needs it: hosts that must not call cudaMalloc or cudaFree once they are running, e.g. a
// real-time audio engine that pre-plans every allocation (the frame loop cannot afford an
// allocator's locks or a device synchronisation), a server whose memory is carved out up front
// by its own pool, or a caller that only owns raw device pointers handed to it by another
// runtime. They pass in their own cache, lengths, inputs and outputs; the split-KV kernel's
// working memory (row plan, rotated q, partial records of streams cut across CTAs) comes from
// the fixed array below instead of from the allocator.
//
// The array is a file-scope __device__ variable: every GPU that loads this library holds its own
// copy, kNoAllocScratchBytes long, until the process exits. Host code cannot use the variable's
// name as a device address, so the first call on each device looks the address up with
// cudaGetSymbolAddress (with that device current) and keeps it for the rest of the process. A
// cudaDeviceReset destroys the context that address belongs to: the entry point must not be
// called on a device after that device was reset.
//
// The stream list is device memory the host never reads, so the checks the allocating path makes
// on the host run in the plan kernel here: a row whose stream index is out of range, that repeats
// an earlier row's stream, or whose position does not fit the capacity is refused. It writes no
// cache row, attends nothing, and its output row is written as zeros; a bit in *err says why.
#include <mutex>
#include <string>

#include "kernels.h"
#include "ptts_b200.h"

namespace {

using namespace ptts;

constexpr int kNoAllocMaxRows = 1024;  // query rows (streams) per call
constexpr int kNoAllocMaxGrid = 160;   // decode CTAs (one per SM; a B200 has 148)
constexpr int kMaxDevices = 64;

constexpr size_t align256(size_t n) { return (n + 255) / 256 * 256; }
constexpr size_t kPlanBytes = align256(sizeof(int32_t) * (3 * kNoAllocMaxRows + 1 + kMaxDecodeGrid));
constexpr size_t kQBytes = align256(sizeof(float) * kNoAllocMaxRows * kRowWidth);
constexpr size_t kPartBytes =
    align256(sizeof(float) * (size_t)(kNoAllocMaxRows + kNoAllocMaxGrid) * (kRowWidth / kHeadDim) * kPartStride);
constexpr size_t kCounterBytes = align256(sizeof(int) * kNoAllocMaxRows * (kRowWidth / kHeadDim));
// About 4.6 MB: plan (12 KB) + rotated q (2 MB) + partial records (2.6 MB) + counters (4 KB).
constexpr size_t kNoAllocScratchBytes = kPlanBytes + kQBytes + kPartBytes + kCounterBytes;

// Shared by every call on a device; it keeps whatever the last call left in it. The plan, the
// rotated q and the partial records are written by each call before it reads them. The merge
// counters must start at zero: each call clears them first (a call cut short by a failed wait
// could have left one set).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct DeviceScratch {
    unsigned char* base = nullptr;
    int grid = 0;
};
std::mutex g_mu;
DeviceScratch g_dev[kMaxDevices];

}  // namespace

// Defined in abi.cu: lets ptts_b200_last_error report this call's message too.
void ptts_b200_set_last_error(const std::string& msg);

extern "C" int ptts_b200_attend_decode_noalloc(void* k_cache, void* v_cache, int num_streams,
                                               int capacity, int kv_dtype, const int32_t* lengths,
                                               const int32_t* streams, int n, const void* q,
                                               const void* k, const void* v, int in_dtype,
                                               int num_kv_heads, float max_period, void* out,
                                               int out_dtype, uint32_t* err, void* cuda_stream) {
    auto refuse = [](int code, const std::string& msg) {
        ptts_b200_set_last_error(msg);
        return code;
    };
    if (!k_cache || !v_cache || !lengths || !streams || !q || !k || !v || !out)
        return refuse(PTTS_B200_ERR_ARG, "a pointer argument is NULL");
    if (n < 1 || n > kNoAllocMaxRows)
        return refuse(PTTS_B200_ERR_ARG, "n = " + std::to_string(n) +
                                             " query rows; the no-alloc decode takes 1.." +
                                             std::to_string(kNoAllocMaxRows) + " per call");
    if (num_streams < 1 || capacity < 1)
        return refuse(PTTS_B200_ERR_ARG, "num_streams and capacity must be positive");
    if ((kv_dtype != PTTS_B200_BF16 && kv_dtype != PTTS_B200_F32) ||
        (in_dtype != PTTS_B200_BF16 && in_dtype != PTTS_B200_F32) ||
        (out_dtype != PTTS_B200_BF16 && out_dtype != PTTS_B200_F32))
        return refuse(PTTS_B200_ERR_ARG, "unknown dtype");
    const int heads = kRowWidth / kHeadDim;
    if (num_kv_heads < 1 || heads % num_kv_heads != 0)
        return refuse(PTTS_B200_ERR_ARG, "the key/value heads do not divide the 8 attention heads");
    if (!(max_period > 1.0f)) return refuse(PTTS_B200_ERR_ARG, "max_period must be above 1");

    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
        return refuse(PTTS_B200_ERR_CUDA, "no current CUDA device");
    DeviceScratch sc;
    {
        // Set-up, once per device, with that device current (the caller's current device).
        std::lock_guard<std::mutex> g(g_mu);
        if (!g_dev[dev].base) {
            void* p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || !p)
                return refuse(PTTS_B200_ERR_CUDA,
                              std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
            int sms = 0;
            e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            if (e != cudaSuccess)
                return refuse(PTTS_B200_ERR_CUDA, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
            g_dev[dev].base = static_cast<unsigned char*>(p);
            g_dev[dev].grid = sms < kNoAllocMaxGrid ? sms : kNoAllocMaxGrid;
        }
        sc = g_dev[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(cuda_stream);
    int32_t* plan_base = reinterpret_cast<int32_t*>(sc.base);
    RowPlan plan;
    plan.row_stream = plan_base;
    plan.row_pos = plan_base + kNoAllocMaxRows;
    plan.row_slot = plan.row_pos;  // no ring here: every row is written at its position
    plan.prefix = plan_base + 2 * kNoAllocMaxRows;
    plan.cta_first = plan.prefix + n + 1;
    float* q_rot = reinterpret_cast<float*>(sc.base + kPlanBytes);
    float* part = reinterpret_cast<float*>(sc.base + kPlanBytes + kQBytes);
    int* counters = reinterpret_cast<int*>(sc.base + kPlanBytes + kQBytes + kPartBytes);
    if (cudaMemsetAsync(counters, 0, sizeof(int) * decode_counter_ints(n), s) != cudaSuccess)
        return refuse(PTTS_B200_ERR_CUDA, "clearing the merge counters failed");

    PlanChecks checks;
    checks.unique = 1;  // n <= 1024
    checks.zero_out = out;
    checks.zero_row_bytes = kRowWidth * (out_dtype == PTTS_B200_BF16 ? 2 : 4);
    launch_plan_decode(lengths, streams, n, num_streams, capacity, plan, RingArgs{}, sc.grid, err, s, checks);
    RopeAppendArgs ra{};
    ra.q = q;
    ra.k = k;
    ra.v = v;
    ra.q_out = q_rot;
    ra.k_cache = k_cache;
    ra.v_cache = v_cache;
    ra.row_stream = plan.row_stream;
    ra.row_pos = plan.row_pos;
    ra.row_slot = plan.row_slot;
    ra.rows = n;
    ra.heads = heads;
    ra.kv_heads = num_kv_heads;
    ra.num_streams = num_streams;
    ra.capacity = capacity;
    for (int i = 0; i < kHeadDim / 2; ++i)  // rope.rs:44-48
        ra.inv_freq[i] = 1.0f / powf(max_period, (float)i / (float)(kHeadDim / 2));
    ra.err = err;
    launch_rope_append(ra, in_dtype == PTTS_B200_BF16, kv_dtype == PTTS_B200_BF16, s);
    DecodeArgs a{};
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.stream_bytes = (long long)capacity * kRowWidth * (kv_dtype == PTTS_B200_BF16 ? 2 : 4);
    a.row_stream = plan.row_stream;
    a.prefix = plan.prefix;
    a.q = q_rot;
    a.out = out;
    a.out_mode = out_dtype == PTTS_B200_BF16 ? kOutBf16 : kOutF32;
    a.part = part;
    a.counters = counters;
    a.B = n;
    a.qscale = (1.0f / sqrtf((float)kHeadDim)) * 1.4426950408889634f;
    a.err = err;
    a.capacity = capacity;  // no ring or windowed stream here (ring_write and window stay null)
    a.cta_first = plan.cta_first;
    a.prestart = true;  // rope_append sits between the plan and this launch
    launch_decode_attn(a, kv_dtype == PTTS_B200_BF16, sc.grid, s);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return refuse(PTTS_B200_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e));
    return PTTS_B200_OK;
}
