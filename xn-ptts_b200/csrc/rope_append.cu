// RoPE on q and k plus the KV-cache append, for the attention op (the model fuses the same
// arithmetic into its in_proj epilogue, see linear.cu).
//
// rope.rs:81-95 / xn rope_i: interleaved pairs (x[2i], x[2i+1]) turned by the f32 angle
// pos * inv_freq[i]; inv_freq comes from the host (rope.rs:44-48, computed there with libm powf
// so the table matches the reference's bit for bit). complete_kv (transformer.rs:84-91) writes
// the rotated k and the v row at the row's position; a KV head is repeated over the
// num_heads / num_kv_heads query heads that share it (transformer.rs:201-211).
#include "common.cuh"
#include "kernels.h"

namespace ptts {
namespace {

template <typename Tin, typename T>
__global__ void rope_append_kernel(RopeAppendArgs a) {
    grid_dep_wait();
    grid_dep_launch();
    const int pairs = kHeadDim / 2;
    const int slots = a.heads + 2 * a.kv_heads;
    const long long total = (long long)a.rows * slots * pairs;
    const long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    if (idx >= total) return;
    const int i = (int)(idx % pairs);
    const int slot = (int)((idx / pairs) % slots);
    const int row = (int)(idx / ((long long)pairs * slots));
    const int sid = a.row_stream[row];
    const int pos = a.row_pos[row], cslot = a.row_slot[row];  // RoPE position, cache slot
    // A row the plan refused (its error bit is set already) writes nothing.
    if (pos == -1 && cslot == -1) return;
    // A windowed stream's position runs past the capacity; its slot never does.
    if (sid < 0 || sid >= a.num_streams || pos < 0 || cslot < 0 || cslot >= a.capacity) {
        set_error(a.err, DEV_ERR_CAPACITY);
        return;
    }
    const Tin* src;
    if (slot < a.heads)
        src = static_cast<const Tin*>(a.q) + ((long long)row * a.heads + slot) * kHeadDim;
    else if (slot < a.heads + a.kv_heads)
        src = static_cast<const Tin*>(a.k) + ((long long)row * a.kv_heads + (slot - a.heads)) * kHeadDim;
    else
        src = static_cast<const Tin*>(a.v) +
              ((long long)row * a.kv_heads + (slot - a.heads - a.kv_heads)) * kHeadDim;
    const float x0 = to_f32(src[2 * i]), x1 = to_f32(src[2 * i + 1]);
    float y0 = x0, y1 = x1;
    if (slot < a.heads + a.kv_heads) {
        float sn, cs;
        sincosf((float)pos * a.inv_freq[i], &sn, &cs);
        y0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        y1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
    }
    if (slot < a.heads) {  // q stays f32 (or f32-grade hi/lo): only this call's attention reads it
        const long long at = ((long long)row * a.heads + slot) * kHeadDim + 2 * i;
        if (a.q_hi) {
            y0 *= a.q_scale;
            y1 *= a.q_scale;
            const uint32_t hi = pack_bf16x2(y0, y1);
            *reinterpret_cast<uint32_t*>(a.q_hi + at) = hi;
            *reinterpret_cast<uint32_t*>(a.q_lo + at) = pack_bf16x2(y0 - bf16lo(hi), y1 - bf16hi(hi));
        } else {
            float* dst = static_cast<float*>(a.q_out) + at;
            dst[0] = y0;
            dst[1] = y1;
        }
        return;
    }
    const bool is_k = slot < a.heads + a.kv_heads;
    const int g = is_k ? slot - a.heads : slot - a.heads - a.kv_heads;
    const int group = a.heads / a.kv_heads;
    T* cache = static_cast<T*>(is_k ? a.k_cache : a.v_cache);
    for (int rep = 0; rep < group; ++rep) {
        T* dst = cache + kv_offset(sid, cslot, g * group + rep, a.num_streams, a.capacity);
        dst[2 * i] = from_f32<T>(y0);
        dst[2 * i + 1] = from_f32<T>(y1);
    }
}

}  // namespace

void launch_rope_append(const RopeAppendArgs& a, bool in_bf16, bool cache_bf16, cudaStream_t s) {
    const long long total = (long long)a.rows * (a.heads + 2 * a.kv_heads) * (kHeadDim / 2);
    const int blocks = (int)((total + 255) / 256);
    if (in_bf16 && cache_bf16)
        launch_k(rope_append_kernel<__nv_bfloat16, __nv_bfloat16>, dim3(blocks), dim3(256), 0, s, a);
    else if (in_bf16)
        launch_k(rope_append_kernel<__nv_bfloat16, float>, dim3(blocks), dim3(256), 0, s, a);
    else if (cache_bf16)
        launch_k(rope_append_kernel<float, __nv_bfloat16>, dim3(blocks), dim3(256), 0, s, a);
    else
        launch_k(rope_append_kernel<float, float>, dim3(blocks), dim3(256), 0, s, a);
}

}  // namespace ptts
