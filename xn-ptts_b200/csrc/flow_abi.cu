// C ABI of the flow head (include/ptts_b200.h, "Flow head"): the keyed weight loader, the time
// embeddings of the solver steps, and the launch sequence of FlowLM::sample_from_noise and of
// one frame (flow_lm.rs:296-324, :360-410; mlp.rs).
#include <cmath>
#include <cstdio>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "host.h"
#include "kernels.h"
#include "ptts_b200.h"

namespace {

using namespace ptts;
using namespace ptts::host;

// f32 -> bf16 bits, round to nearest even (finite inputs).
uint16_t bf16_bits(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}
float bf16_value(uint16_t h) {
    const uint32_t u = (uint32_t)h << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// A tensor-core linear of the flow net: weights [n][k] as bf16 hi and (when any is nonzero) lo
// planes, f32 bias.
struct DenseLinear {
    DevBuf hi, lo, bias;
    bool has_lo = false;
    int n = 0, k = 0;
    void upload(const std::vector<float>& w, const std::vector<float>& b, int n_, int k_) {
        n = n_;
        k = k_;
        std::vector<uint16_t> h(w.size()), l(w.size());
        has_lo = false;
        for (size_t i = 0; i < w.size(); ++i) {
            h[i] = bf16_bits(w[i]);
            l[i] = bf16_bits(w[i] - bf16_value(h[i]));
            has_lo = has_lo || (l[i] & 0x7FFFu) != 0;
        }
        CK(cudaMemcpy(hi.need(h.size() * 2), h.data(), h.size() * 2, cudaMemcpyHostToDevice));
        if (has_lo) CK(cudaMemcpy(lo.need(l.size() * 2), l.data(), l.size() * 2, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(bias.need(b.size() * 4), b.data(), b.size() * 4, cudaMemcpyHostToDevice));
    }
};

void put(DevBuf& d, const std::vector<float>& v) {
    CK(cudaMemcpy(d.need(v.size() * 4), v.data(), v.size() * 4, cudaMemcpyHostToDevice));
}

}  // namespace

struct ptts_b200_flow {
    int device;
    ptts_b200_flow_config cfg;
    int time_conds;
    std::map<std::string, size_t> expected;          // name -> numel
    std::map<std::string, std::vector<float>> host;  // tensors set so far
    bool ready = false;
    // device weights
    DevBuf input_linear, condition, bos, out_norm_w, out_norm_b, eos_w;
    float eos_b = 0.f;
    bool has_condition = false;
    DevBuf in_proj_w, in_proj_b, final_w, final_b, temb;
    DenseLinear cond, ada;
    std::vector<std::unique_ptr<DenseLinear>> lin1, lin2;
    std::vector<std::unique_ptr<DevBuf>> ln_w, ln_b;
    DevBuf err;
    // workspace, sized for `rows` rows
    int rows = 0;
    DevBuf x_in, hidden, t_hi, t_lo, y_hi, y_lo, ada_out, xf, h_hi, h_lo, h1_hi, h1_lo, hf, cur_a, cur_b;

    uint64_t uid = 0;  // distinguishes a new flow head at a recycled address
    int gen = 0;       // bumped whenever the workspace moves (a recorded frame graph is then stale)
    int ada_width() const { return cfg.flow_dim * (3 * cfg.flow_depth + 2); }
    void size(int n) {
        if (n <= rows) return;
        ++gen;
        const size_t d = cfg.d_model, C = cfg.flow_dim, L = cfg.ldim;
        x_in.need(n * d * 2);
        hidden.need(n * d * 4);
        t_hi.need(n * d * 2);
        t_lo.need(n * d * 2);
        y_hi.need(n * C * 2);
        y_lo.need(n * C * 2);
        ada_out.need((size_t)n * ada_width() * 4);
        xf.need(n * C * 4);
        h_hi.need(n * C * 2);
        h_lo.need(n * C * 2);
        h1_hi.need(n * C * 2);
        h1_lo.need(n * C * 2);
        hf.need(n * C * 4);
        cur_a.need(n * L * 4);
        cur_b.need(n * L * 4);
        rows = n;
    }
};

namespace {

void check_flow(const ptts_b200_flow* f, bool need_ready = true) {
    require(f != nullptr, PTTS_B200_ERR_ARG, "flow is NULL");
    require(!need_ready || f->ready, PTTS_B200_ERR_STATE, "flow weights not finished (ptts_b200_flow_finish)");
}

const std::vector<float>& tensor(ptts_b200_flow* f, const std::string& name) {
    auto it = f->host.find(name);
    require(it != f->host.end(), PTTS_B200_ERR_STATE, "flow tensor missing: " + name);
    return it->second;
}

// SimpleMLPAdaLN::time_embedding (mlp.rs:204-211) of the times (s, t) through TimestepEmbedder
// (mlp.rs:54-81): cat(cos, sin)(time * freqs) -> linear1 -> SiLU -> linear2 -> RMS norm * alpha,
// averaged over the embedders. Host f64, once per flow.
std::vector<float> time_embedding(ptts_b200_flow* f, const double* times) {
    const int C = f->cfg.flow_dim, F = f->cfg.freq_dim;
    std::vector<double> acc(C, 0.0);
    for (int e = 0; e < f->time_conds; ++e) {
        const std::string p = "flow_net.time_embed." + std::to_string(e) + ".";
        const auto& freqs = tensor(f, p + "freqs");
        const auto& w1 = tensor(f, p + "mlp.0.weight");
        const auto& b1 = tensor(f, p + "mlp.0.bias");
        const auto& w2 = tensor(f, p + "mlp.2.weight");
        const auto& b2 = tensor(f, p + "mlp.2.bias");
        const auto& alpha = tensor(f, p + "mlp.3.alpha");
        std::vector<double> emb(F), h(C), y(C);
        for (int j = 0; j < F / 2; ++j) {
            const double a = (double)(float)(times[e] * freqs[j]);
            emb[j] = std::cos(a);
            emb[F / 2 + j] = std::sin(a);
        }
        for (int o = 0; o < C; ++o) {
            double s = b1[o];
            for (int k = 0; k < F; ++k) s += (double)w1[(size_t)o * F + k] * emb[k];
            h[o] = s / (1.0 + std::exp(-s));
        }
        for (int o = 0; o < C; ++o) {
            double s = b2[o];
            for (int k = 0; k < C; ++k) s += (double)w2[(size_t)o * C + k] * h[k];
            y[o] = s;
        }
        double denom;
        if (f->cfg.time_norm == PTTS_B200_TIME_RMS) {
            double ms = 0.0;
            for (double v : y) ms += v * v;
            denom = std::sqrt(ms / C + 1e-5);
        } else {  // centred, unbiased variance (torch.var)
            double mean = 0.0, var = 0.0;
            for (double v : y) mean += v;
            mean /= C;
            for (double v : y) var += (v - mean) * (v - mean);
            denom = std::sqrt(var / (C - 1) + 1e-5);
        }
        for (int o = 0; o < C; ++o) acc[o] += y[o] / denom * alpha[o];
    }
    std::vector<float> out(C);
    for (int o = 0; o < C; ++o) out[o] = (float)(acc[o] / f->time_conds);
    return out;
}

void gemm(const ptts_b200_flow* f, LinearEpi epi, int rows, const void* a_hi, const void* a_lo,
          const DenseLinear& w, float* y, void* yb, void* yb_lo, const float* aux, int aux_stride,
          cudaStream_t s) {
    LinearArgs a{};
    a.M = rows;
    a.N = w.n;
    a.K = w.k;
    a.splits = 1;
    a.a = a_hi;
    a.a_lo = a_lo;
    a.a_f16 = 0;
    a.wh = w.hi.p;
    a.wh_lo = w.has_lo ? w.lo.p : nullptr;
    a.scale = nullptr;
    a.bias = w.bias.as<float>();
    a.aux = aux;
    a.aux_stride = aux_stride;
    a.y = y;
    a.yb = yb;
    a.yb_lo = yb_lo;
    a.err = f->err.as<uint32_t>();
    require(launch_linear_tc(a, epi, s), PTTS_B200_ERR_UNSUPPORTED,
            "flow linear " + std::to_string(w.n) + "x" + std::to_string(w.k) + " has no tensor-core kernel");
    CK(cudaGetLastError());
}

// FlowLM::sample_from_noise from `src` rows [n][d_model] f32: out_norm first when `normalise`
// (the backbone output), else `src` is already t_out. The rows use workspace rows row_off ..
// row_off + n - 1, so calls on disjoint row ranges may run at the same time (the two lanes of a
// frame); the workspace must already hold row_off + n rows.
void sample(ptts_b200_flow* f, const float* src, bool normalise, int n, const float* noise, float* latent,
            float* eos, cudaStream_t s, int row_off = 0) {
    const auto& c = f->cfg;
    const int C = c.flow_dim, L = c.ldim, W = f->ada_width();
    if (row_off == 0) f->size(n);
    require(row_off + n <= f->rows, PTTS_B200_ERR_STATE, "flow workspace smaller than the rows asked for");
    const size_t o = (size_t)row_off;
    __nv_bfloat16* t_hi = f->t_hi.as<__nv_bfloat16>() + o * c.d_model;
    __nv_bfloat16* t_lo = f->t_lo.as<__nv_bfloat16>() + o * c.d_model;
    __nv_bfloat16* y_hi = f->y_hi.as<__nv_bfloat16>() + o * C;
    __nv_bfloat16* y_lo = f->y_lo.as<__nv_bfloat16>() + o * C;
    float* ada = f->ada_out.as<float>() + o * W;
    float* xf = f->xf.as<float>() + o * C;
    __nv_bfloat16* h_hi = f->h_hi.as<__nv_bfloat16>() + o * C;
    __nv_bfloat16* h_lo = f->h_lo.as<__nv_bfloat16>() + o * C;
    __nv_bfloat16* h1_hi = f->h1_hi.as<__nv_bfloat16>() + o * C;
    __nv_bfloat16* h1_lo = f->h1_lo.as<__nv_bfloat16>() + o * C;
    float* hf = f->hf.as<float>() + o * C;
    float* cur_a = f->cur_a.as<float>() + o * L;
    float* cur_b = f->cur_b.as<float>() + o * L;
    FlowNormArgs na{};
    na.M = n;
    na.d = c.d_model;
    na.x = src;
    na.gamma = normalise ? f->out_norm_w.as<float>() : nullptr;
    na.beta = normalise ? f->out_norm_b.as<float>() : nullptr;
    na.eps = 1e-5f;
    na.eos_w = f->eos_w.as<float>();
    na.eos_b = f->eos_b;
    na.eos = eos;
    na.hi = t_hi;
    na.lo = t_lo;
    launch_flow_norm_eos(na, s);
    CK(cudaGetLastError());
    const int steps = c.flow_type == PTTS_B200_FLOW_LSD ? c.lsd_steps : 1;
    const float* cur = noise;
    for (int i = 0; i < steps; ++i) {
        // x = input_proj(current)
        FlowSmallArgs ip{};
        ip.M = n;
        ip.N = C;
        ip.K = L;
        ip.a = cur;
        ip.w = f->in_proj_w.as<float>();
        ip.bias = f->in_proj_b.as<float>();
        ip.y = xf;
        launch_flow_small(ip, s);
        CK(cudaGetLastError());
        // y_act = silu(cond_embed(t_out) + t_emb): one linear, both biases in its epilogue
        if (f->time_conds > 0)
            gemm(f, EPI_COND, n, t_hi, t_lo, f->cond, nullptr, y_hi, y_lo, f->temb.as<float>() + (size_t)i * C, 0, s);
        else
            gemm(f, EPI_BIAS_SILU, n, t_hi, t_lo, f->cond, nullptr, y_hi, y_lo, nullptr, 0, s);
        // every block's adaLN modulation (and the final layer's) in one linear
        gemm(f, EPI_BIAS, n, y_hi, y_lo, f->ada, ada, nullptr, nullptr, nullptr, 0, s);
        for (int b = 0; b < c.flow_depth; ++b) {
            FlowModArgs m{};
            m.M = n;
            m.C = C;
            m.x = xf;
            m.gamma = f->ln_w[b]->as<float>();
            m.beta = f->ln_b[b]->as<float>();
            m.eps = 1e-6f;
            m.shift = ada + (size_t)b * 3 * C;
            m.scale = ada + (size_t)b * 3 * C + C;
            m.stride = W;
            m.hi = h_hi;
            m.lo = h_lo;
            launch_flow_ln_mod(m, s);
            CK(cudaGetLastError());
            gemm(f, EPI_BIAS_SILU, n, h_hi, h_lo, *f->lin1[b], nullptr, h1_hi, h1_lo, nullptr, 0, s);
            gemm(f, EPI_GATE_RESID, n, h1_hi, h1_lo, *f->lin2[b], xf, nullptr, nullptr,
                 ada + (size_t)b * 3 * C + 2 * C, W, s);
        }
        FlowModArgs m{};
        m.M = n;
        m.C = C;
        m.x = xf;
        m.eps = 1e-6f;
        m.shift = ada + (size_t)c.flow_depth * 3 * C;
        m.scale = ada + (size_t)c.flow_depth * 3 * C + C;
        m.stride = W;
        FlowOutArgs o{};
        o.M = n;
        o.C = C;
        o.L = L;
        o.h = hf;
        o.w = f->final_w.as<float>();
        o.bias = f->final_b.as<float>();
        o.cur = c.flow_type == PTTS_B200_FLOW_DRIFTING ? nullptr : cur;
        o.step_scale = c.flow_type == PTTS_B200_FLOW_LSD ? 1.0f / (float)steps : 1.0f;
        float* next = i + 1 == steps ? latent : (i % 2 == 0 ? cur_a : cur_b);
        o.out = next;
        if (!launch_flow_final(m, o, s)) {  // other shapes: the modulated rows through memory
            m.y = hf;
            launch_flow_ln_mod(m, s);
            CK(cudaGetLastError());
            launch_flow_out(o, s);
        }
        CK(cudaGetLastError());
        cur = next;
    }
}

}  // namespace

// ---- pieces of ptts_b200_frame (abi.cu records them with the step in one CUDA graph) ---------

// The flow head is ready for `n` rows: its workspace sized (outside any capture). Returns what
// a recorded frame graph depends on: the object's identity and its workspace generation.
uint64_t ptts_b200_flow_prepare(ptts_b200_flow* f, int n, int d_model) {
    check_flow(f);
    require(f->cfg.d_model == d_model, PTTS_B200_ERR_STATE, "the flow head and the model differ in d_model");
    DeviceScope scope(f->device);
    f->size(n);
    return (f->uid << 32) | (uint64_t)(uint32_t)f->gen;
}
int ptts_b200_flow_ldim(const ptts_b200_flow* f) { return f->cfg.ldim; }

// input_linear(latent) (+ condition) -> the backbone's bf16 input rows x [n][d_model]; latent
// nullptr: every row from bos_emb (StepInput::Bos).
void ptts_b200_flow_input(ptts_b200_flow* f, const float* latent, __nv_bfloat16* x, int n, cudaStream_t s) {
    FlowSmallArgs in{};
    in.M = n;
    in.N = f->cfg.d_model;
    in.K = f->cfg.ldim;
    in.a = latent;
    in.a_row = f->bos.as<float>();
    in.w = f->input_linear.as<float>();
    in.add = f->has_condition ? f->condition.as<float>() : nullptr;
    in.yb = x;
    launch_flow_small(in, s);
    CK(cudaGetLastError());
}

// out_norm of the backbone's output rows, then sample_from_noise, for rows row_off ..
// row_off + n - 1 of the frame (the pointers are those rows' own; the workspace rows match).
void ptts_b200_flow_head(ptts_b200_flow* f, const float* hidden, int n, const float* noise, float* latent,
                         float* eos, cudaStream_t s, int row_off) {
    sample(f, hidden, true, n, noise, latent, eos, s, row_off);
}

// Whether `name` is one of this flow head's tensors (for the GGUF loader, gguf.cu).
bool ptts_b200_flow_wants(const ptts_b200_flow* flow, const std::string& name) {
    return flow && (name == "condition" || flow->expected.count(name) != 0);
}

extern "C" {

int ptts_b200_flow_create(int device, const ptts_b200_flow_config* config, ptts_b200_flow** out) {
    return guarded([&] {
        require(config && out, PTTS_B200_ERR_ARG, "NULL argument");
        const ptts_b200_flow_config& c = *config;
        auto wide = [](int v) { return v == 128 || v == 256 || v == 512 || v == 1024; };
        require(wide(c.d_model), PTTS_B200_ERR_UNSUPPORTED, "d_model must be 128, 256, 512 or 1024");
        require(wide(c.flow_dim), PTTS_B200_ERR_UNSUPPORTED, "flow_dim must be 128, 256, 512 or 1024");
        require(c.flow_depth >= 1, PTTS_B200_ERR_ARG, "flow_depth must be >= 1");
        require(c.ldim >= 1 && c.ldim <= 64, PTTS_B200_ERR_UNSUPPORTED, "ldim must be in 1..64");
        require((size_t)c.flow_dim * (c.ldim + 1) * 4 <= 200 * 1024, PTTS_B200_ERR_UNSUPPORTED,
                "flow_dim x (ldim + 1) floats must fit the final layer's 200 KB of shared memory");
        require((size_t)c.flow_dim * c.ldim * 4 <= 200 * 1024, PTTS_B200_ERR_UNSUPPORTED,
                "flow_dim * ldim too large for the final layer's kernel");
        require(c.flow_type >= 0 && c.flow_type <= 2, PTTS_B200_ERR_ARG, "unknown flow_type");
        require(c.flow_type != PTTS_B200_FLOW_LSD || c.lsd_steps >= 1, PTTS_B200_ERR_ARG, "lsd_steps must be >= 1");
        require(c.flow_type != PTTS_B200_FLOW_LSD || (c.freq_dim >= 2 && c.freq_dim % 2 == 0), PTTS_B200_ERR_ARG,
                "freq_dim must be even");
        require(c.time_norm == PTTS_B200_TIME_RMS || c.time_norm == PTTS_B200_TIME_RMS_VAR, PTTS_B200_ERR_ARG,
                "unknown time_norm");
        int count = 0;
        CK(cudaGetDeviceCount(&count));
        require(device >= 0 && device < count, PTTS_B200_ERR_ARG, "no such device");
        static uint64_t next_uid = 1;
        auto f = std::make_unique<ptts_b200_flow>();
        f->uid = next_uid++;
        f->device = device;
        f->cfg = c;
        f->time_conds = c.flow_type == PTTS_B200_FLOW_LSD ? 2 : 0;
        const size_t d = c.d_model, C = c.flow_dim, L = c.ldim, F = c.freq_dim;
        auto& e = f->expected;
        e["input_linear.weight"] = d * L;
        e["out_norm.weight"] = d;
        e["out_norm.bias"] = d;
        e["out_eos.weight"] = d;
        e["out_eos.bias"] = 1;
        e["bos_emb"] = L;
        e["flow_net.input_proj.weight"] = C * L;
        e["flow_net.input_proj.bias"] = C;
        e["flow_net.cond_embed.weight"] = C * d;
        e["flow_net.cond_embed.bias"] = C;
        for (int i = 0; i < f->time_conds; ++i) {
            const std::string p = "flow_net.time_embed." + std::to_string(i) + ".";
            e[p + "freqs"] = F / 2;
            e[p + "mlp.0.weight"] = C * F;
            e[p + "mlp.0.bias"] = C;
            e[p + "mlp.2.weight"] = C * C;
            e[p + "mlp.2.bias"] = C;
            e[p + "mlp.3.alpha"] = C;
        }
        for (int b = 0; b < c.flow_depth; ++b) {
            const std::string p = "flow_net.res_blocks." + std::to_string(b) + ".";
            e[p + "in_ln.weight"] = C;
            e[p + "in_ln.bias"] = C;
            e[p + "mlp.0.weight"] = C * C;
            e[p + "mlp.0.bias"] = C;
            e[p + "mlp.2.weight"] = C * C;
            e[p + "mlp.2.bias"] = C;
            e[p + "adaLN_modulation.1.weight"] = 3 * C * C;
            e[p + "adaLN_modulation.1.bias"] = 3 * C;
        }
        e["flow_net.final_layer.adaLN_modulation.1.weight"] = 2 * C * C;
        e["flow_net.final_layer.adaLN_modulation.1.bias"] = 2 * C;
        e["flow_net.final_layer.linear.weight"] = L * C;
        e["flow_net.final_layer.linear.bias"] = L;
        *out = f.release();
    });
}

void ptts_b200_flow_destroy(ptts_b200_flow* flow) {
    if (!flow) return;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(flow->device);
    delete flow;
    if (prev >= 0) cudaSetDevice(prev);
}

int ptts_b200_flow_set_tensor(ptts_b200_flow* flow, const char* name, const float* host, int64_t numel) {
    return guarded([&] {
        check_flow(flow, false);
        require(name && host, PTTS_B200_ERR_ARG, "NULL argument");
        const std::string key(name);
        size_t want = 0;
        if (key == "condition") {
            want = flow->cfg.d_model;
        } else {
            auto it = flow->expected.find(key);
            require(it != flow->expected.end(), PTTS_B200_ERR_ARG, "unknown flow tensor: " + key);
            want = it->second;
        }
        require(numel == (int64_t)want, PTTS_B200_ERR_ARG,
                key + ": " + std::to_string(numel) + " elements, expected " + std::to_string(want));
        flow->host[key].assign(host, host + numel);
        flow->ready = false;
    });
}

int ptts_b200_flow_finish(ptts_b200_flow* flow) {
    return guarded([&] {
        check_flow(flow, false);
        for (const auto& kv : flow->expected)
            require(flow->host.count(kv.first) != 0, PTTS_B200_ERR_STATE, "flow tensor missing: " + kv.first);
        DeviceScope scope(flow->device);
        const auto& c = flow->cfg;
        const int C = c.flow_dim, d = c.d_model;
        put(flow->input_linear, tensor(flow, "input_linear.weight"));
        flow->has_condition = flow->host.count("condition") != 0;
        if (flow->has_condition) put(flow->condition, tensor(flow, "condition"));
        put(flow->bos, tensor(flow, "bos_emb"));
        put(flow->out_norm_w, tensor(flow, "out_norm.weight"));
        put(flow->out_norm_b, tensor(flow, "out_norm.bias"));
        put(flow->eos_w, tensor(flow, "out_eos.weight"));
        flow->eos_b = tensor(flow, "out_eos.bias")[0];
        put(flow->in_proj_w, tensor(flow, "flow_net.input_proj.weight"));
        put(flow->in_proj_b, tensor(flow, "flow_net.input_proj.bias"));
        put(flow->final_w, tensor(flow, "flow_net.final_layer.linear.weight"));
        put(flow->final_b, tensor(flow, "flow_net.final_layer.linear.bias"));
        flow->cond.upload(tensor(flow, "flow_net.cond_embed.weight"), tensor(flow, "flow_net.cond_embed.bias"), C, d);
        std::vector<float> aw, ab;
        flow->lin1.clear();
        flow->lin2.clear();
        flow->ln_w.clear();
        flow->ln_b.clear();
        for (int b = 0; b < c.flow_depth; ++b) {
            const std::string p = "flow_net.res_blocks." + std::to_string(b) + ".";
            const auto& w = tensor(flow, p + "adaLN_modulation.1.weight");
            const auto& bb = tensor(flow, p + "adaLN_modulation.1.bias");
            aw.insert(aw.end(), w.begin(), w.end());
            ab.insert(ab.end(), bb.begin(), bb.end());
            flow->lin1.push_back(std::make_unique<DenseLinear>());
            flow->lin1.back()->upload(tensor(flow, p + "mlp.0.weight"), tensor(flow, p + "mlp.0.bias"), C, C);
            flow->lin2.push_back(std::make_unique<DenseLinear>());
            flow->lin2.back()->upload(tensor(flow, p + "mlp.2.weight"), tensor(flow, p + "mlp.2.bias"), C, C);
            flow->ln_w.push_back(std::make_unique<DevBuf>());
            put(*flow->ln_w.back(), tensor(flow, p + "in_ln.weight"));
            flow->ln_b.push_back(std::make_unique<DevBuf>());
            put(*flow->ln_b.back(), tensor(flow, p + "in_ln.bias"));
        }
        const auto& fw = tensor(flow, "flow_net.final_layer.adaLN_modulation.1.weight");
        const auto& fb = tensor(flow, "flow_net.final_layer.adaLN_modulation.1.bias");
        aw.insert(aw.end(), fw.begin(), fw.end());
        ab.insert(ab.end(), fb.begin(), fb.end());
        flow->ada.upload(aw, ab, flow->ada_width(), C);
        // lsd_time_embeddings (flow_lm.rs:84-98): step i is conditioned on (i / N, (i + 1) / N).
        if (flow->time_conds > 0) {
            const int N = c.lsd_steps;
            std::vector<float> all;
            for (int i = 0; i < N; ++i) {
                const double times[2] = {(double)((float)i / (float)N), (double)((float)(i + 1) / (float)N)};
                const std::vector<float> t = time_embedding(flow, times);
                all.insert(all.end(), t.begin(), t.end());
            }
            put(flow->temb, all);
        }
        flow->err.need_zeroed(sizeof(uint32_t));
        CK(cudaDeviceSynchronize());
        flow->ready = true;
    });
}

int ptts_b200_flow_sample(ptts_b200_flow* flow, const float* t_out, int n, const float* noise, float* latent,
                          float* eos, void* cuda_stream) {
    return guarded([&] {
        check_flow(flow);
        require(t_out && noise && latent && eos, PTTS_B200_ERR_ARG, "NULL argument");
        require(n >= 1, PTTS_B200_ERR_ARG, "n must be >= 1");
        DeviceScope scope(flow->device);
        sample(flow, t_out, false, n, noise, latent, eos, static_cast<cudaStream_t>(cuda_stream));
    });
}

}  // extern "C"
