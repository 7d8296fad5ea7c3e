// decoder.cu — the Mica decoder behind include/laya_decoder.h: weights, workspace and the order of kernels of one
// prefill (Qwen35Model.Forward, Mica/Models/Qwen35Model.cs:462-532) with every projection a Q8_0 product
// (q8_gemm.cu) and the rest in decoder_kernels.cu.
//
// Device state:
//   weights     per layer the stacked Q8_0 projections (fp16-held codes [N, K], block scales [K/32, ldw]) — DeltaNet
//               in_proj [qkv | z | b | a] and out_proj, or attention [q·gate | k | v] and o_proj; MLP [gate | up]
//               and down — plus the fp32 norms (1 + w), conv taps [K, conv_dim], −exp(A_log), dt_bias; the Q8_0
//               token table [vocab, hidden] serves the embedding rows and the tied head.
//   workspace   sized for max_tokens rows: the residual stream x [T, h] fp32; one projection output [T, widest];
//               the DeltaNet conv/q/k/v [T, conv_dim] and core [T, value_dim]; fp16 q/k/v of full attention; the
//               activation codes of the next product [T, widest K] with scales [widest K/32, ldx]; β and decay.
//   inputs      ids, row → sequence, sequence starts and lengths, the 64-query tiles of full attention and the label
//               ids travel in one pinned staging buffer and one host→device copy per forward.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "../../include/laya_b200.h"
#include "../../include/laya_decoder.h"
#include "common.cuh"
#include "decoder.h"
#include "internal.h"

using namespace laya;

namespace {

#define RC(x)                      \
    do {                           \
        int rc_ = (x);             \
        if (rc_ != OK) return rc_; \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

int rup(int x, int m) { return (x + m - 1) / m * m; }

float half_bits(uint16_t b) {
    __half h;
    memcpy(&h, &b, 2);
    return __half2float(h);
}
float bf16_bits(uint16_t b) {
    const uint32_t u = static_cast<uint32_t>(b) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

// A Q8_0 matrix whose rows may be filled piecewise (the stacked projections).
struct QMat {
    q8::code_t* q = nullptr;
    float* d = nullptr;
    int N = 0, K = 0, ldw = 0;
};

// A checkpoint tensor that fills rows of a stacked Q8_0 matrix: rows [row0, row0 + rows), or — `interleaved` — its
// 32-row groups g at rows 64g + row0 .. 64g + row0 + 31 (the MLP's [32 gate | 32 up] groups, row0 = 0 or 32).
struct Part {
    QMat* m;
    int row0, rows;
    bool interleaved = false;
};

struct Layer {
    int kind = LAYA_DECODER_LINEAR;
    QMat mix_in, mix_out, gate_up, down;   // in_proj | qkv; out_proj | o_proj; MLP
    float *in_norm = nullptr, *post_norm = nullptr;
    float *conv_w = nullptr, *neg_a = nullptr, *dt_bias = nullptr, *gnorm = nullptr;   // DeltaNet
    float *qnorm = nullptr, *knorm = nullptr;                                         // full attention
};

// Vector parameters: destination and the transform applied on upload.
enum VecKind { V_PLAIN = 0, V_ONE_PLUS = 1, V_NEG_EXP = 2, V_CONV = 3 };
struct Vec {
    float** dst;
    int64_t count;
    VecKind kind;
};

}  // namespace

struct laya_decoder {
    int device = 0;
    cudaStream_t own = nullptr, stream = nullptr;
    laya_decoder_desc d{};
    std::vector<int> kinds;
    int* err = nullptr;

    // geometry
    int cd = 0, key_dim = 0, vd = 0, nin = 0, ld_in = 0, q_width = 0, nqkv = 0, half = 0, maxK = 0, ldx = 0,
        widest = 0, core_w = 0;

    std::vector<Layer> layers;
    QMat table;
    float* final_norm = nullptr;
    std::map<std::string, Part> parts;
    std::map<std::string, Vec> vecs;
    std::set<std::string> have;

    // workspace
    float *x = nullptr, *big = nullptr, *conv = nullptr, *core = nullptr, *beta = nullptr, *decay = nullptr,
          *mix = nullptr;
    __half *q16 = nullptr, *k16 = nullptr, *v16 = nullptr;
    q8::code_t *qa = nullptr, *qa2 = nullptr;   // activation codes of the next product; qa2: the down projection's
    float *da = nullptr, *da2 = nullptr;
    float *cosv = nullptr, *sinv = nullptr;
    // readout
    float *hid = nullptr, *dlast = nullptr, *logit_buf = nullptr;
    q8::code_t* qlast = nullptr;
    int ldl = 0, logit_cap = 0;
    // inputs
    int32_t* in_dev = nullptr;
    int32_t* in_host = nullptr;
    size_t in_cap = 0;
    cudaEvent_t in_done = nullptr;
    bool in_pending = false;
    int32_t *ids = nullptr, *tok_seq = nullptr, *seq_start = nullptr, *seq_len = nullptr, *last_row = nullptr,
            *tile_seq = nullptr, *tile_p0 = nullptr, *labels = nullptr;
    int n_tiles = 0;
    // the states of the current forward: positions already read, checkpoints, and the pointer tables
    // ptrs [2·layers·n_seq]: per layer two rows of one entry per sequence (full: keys, values; DeltaNet: conv tail,
    // recurrent state — 0 without a state), then [2·layers·n_snap] the same for the snapshots
    int32_t *pos0 = nullptr, *snap_begin = nullptr, *snap_at = nullptr;
    int32_t *lt_seq = nullptr, *lt_p0 = nullptr;   // the attention tile holding each sequence's last row
    float *xl = nullptr, *corel = nullptr;         // the last layer's readout rows: residual and attention output
    uint64_t* ptrs = nullptr;
    int cur_seqs = 0, cur_snaps = 0;
    bool with_states = false;
    int rope_cap = 0;
    std::set<laya_decoder_state*> states;
    std::set<laya_decoder_mark*> marks;
    cudaMemPool_t pool = nullptr;   // state and mark blocks: freed blocks stay in the pool for the next request

    // profiling: 0 products, 1 delta rule, 2 full attention
    bool profiling = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev_pool;
    std::vector<std::pair<int, double>> ev_work;
    double prof_ms[3] = {0, 0, 0}, prof_ops[3] = {0, 0, 0};
    long long prof_n[3] = {0, 0, 0};

    bool chunked_rule = false;   // stateless reads: the delta rule in 64-token chunks where it applies (opt-in)

    // recorder: name → (buffer, capacity in floats, floats of the last copy)
    bool record = false;
    struct Recorded { float* p = nullptr; size_t cap = 0, count = 0; };
    std::map<std::string, Recorded> rec;

    std::vector<void*> allocs;
};

// Qwen35State in device memory: one stream-ordered block — first the fixed part (per DeltaNet layer its conv tail
// [K−1, cd] and recurrent state [vh, dk, dv], fp32), then per full-attention layer keys and values
// [capacity, kv·hd] fp16.  dec is cleared when the decoder goes first (the block is freed with it).
struct laya_decoder_state {
    laya_decoder* dec = nullptr;
    int capacity = 0, length = 0;
    char* block = nullptr;
    size_t fixed = 0, bytes = 0;
    std::vector<float*> tail, rec;
    std::vector<__half*> k, v;
};
// Qwen35State.Mark: the length and a copy of the fixed part.
struct laya_decoder_mark {
    laya_decoder* dec = nullptr;
    int length = 0;
    char* block = nullptr;
    size_t bytes = 0;
};

namespace {

int dalloc(laya_decoder* c, void** p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    c->allocs.push_back(*p);
    return OK;
}
template <class T>
int dalloc_t(laya_decoder* c, T** p, size_t count) {
    return dalloc(c, reinterpret_cast<void**>(p), count * sizeof(T));
}

int alloc_qmat(laya_decoder* c, QMat& m, int N, int K) {
    m.N = N; m.K = K; m.ldw = rup(N, 128);
    RC(dalloc_t(c, &m.q, static_cast<size_t>(N) * K));
    RC(dalloc_t(c, &m.d, static_cast<size_t>(K / 32) * m.ldw));
    LAYA_CUDA(cudaMemsetAsync(m.d, 0, sizeof(float) * static_cast<size_t>(K / 32) * m.ldw, c->stream));
    return OK;
}

template <class F>
int timed(laya_decoder* c, int kind, double ops, F&& launch) {
    if (!c->profiling) return launch();
    if (c->ev_work.size() == c->ev_pool.size()) {
        cudaEvent_t e0, e1;
        LAYA_CUDA(cudaEventCreate(&e0));
        LAYA_CUDA(cudaEventCreate(&e1));
        c->ev_pool.push_back({e0, e1});
    }
    auto& ev = c->ev_pool[c->ev_work.size()];
    LAYA_CUDA(cudaEventRecord(ev.first, c->stream));
    const int rc = launch();
    LAYA_CUDA(cudaEventRecord(ev.second, c->stream));
    c->ev_work.push_back({kind, ops});
    return rc;
}

int collect_profile(laya_decoder* c) {
    if (c->ev_work.empty()) return OK;
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    for (size_t i = 0; i < c->ev_work.size(); ++i) {
        float ms = 0;
        LAYA_CUDA(cudaEventElapsedTime(&ms, c->ev_pool[i].first, c->ev_pool[i].second));
        const int k = c->ev_work[i].first;
        c->prof_ms[k] += ms;
        c->prof_ops[k] += c->ev_work[i].second;
        c->prof_n[k] += 1;
    }
    c->ev_work.clear();
    return OK;
}

int check_device_error(laya_decoder* c) {
    int h = 0;
    LAYA_CUDA(cudaMemcpyAsync(&h, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    if (h != 0) {
        LAYA_CUDA(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream));
        LAYA_CUDA(cudaStreamSynchronize(c->stream));
        if (h == LAYA_DEV_ERR_TIMEOUT) { set_error("a device-side wait timed out"); return ERR_DEVICE_TIMEOUT; }
        set_error("token id outside the vocabulary");
        return ERR_OUT_OF_RANGE;
    }
    return OK;
}

int record_copy(laya_decoder* c, const std::string& name, const float* src, size_t count) {
    if (!c->record) return OK;
    auto& b = c->rec[name];
    if (b.cap < count) {
        if (b.p) cudaFree(b.p);
        b.p = nullptr;
        LAYA_CUDA(cudaMalloc(&b.p, count * sizeof(float)));
        b.cap = count;
    }
    b.count = count;
    LAYA_CUDA(cudaMemcpyAsync(b.p, src, count * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    return OK;
}

template <class T>
T* const* seq_table(laya_decoder* c, int layer, int which) {
    return reinterpret_cast<T* const*>(c->ptrs + (2 * static_cast<size_t>(layer) + which) * c->cur_seqs);
}
template <class T>
T* const* snap_table(laya_decoder* c, int layer, int which) {
    return reinterpret_cast<T* const*>(c->ptrs + 2 * static_cast<size_t>(c->d.layers) * c->cur_seqs +
                                       (2 * static_cast<size_t>(layer) + which) * c->cur_snaps);
}

// y = Q8(x) · Wᵀ with the codes of x in (qx, dx).
int product_from(laya_decoder* c, const QMat& w, int T, int epi, float* out, int ldo, const q8::code_t* qx,
                 const float* dx) {
    q8::GemmArgs a{};
    a.M = T; a.N = w.N; a.K = w.K;
    a.qx = qx; a.dx = dx; a.ldx = c->ldx;
    a.qw = w.q; a.dw = w.d; a.ldw = w.ldw;
    a.epi = epi;
    a.out = out; a.ldo = ldo;
    a.err = c->err;
    return timed(c, 0, 2.0 * T * static_cast<double>(w.N) * w.K, [&] { return q8::gemm(a, c->stream); });
}
int product(laya_decoder* c, const QMat& w, int T, int epi, float* out, int ldo) {
    return product_from(c, w, T, epi, out, ldo, c->qa, c->da);
}

int rms_codes(laya_decoder* c, const float* scale, int T, const float* x = nullptr) {
    dec::RmsArgs r{};
    r.rows = T; r.n = c->d.hidden; r.x = x ? x : c->x; r.scale = scale; r.eps = c->d.eps;
    r.q = c->qa; r.d = c->da; r.ldd = c->ldx;
    return dec_rms_q8(r, c->stream);
}

// The mixer's output goes into the residual stream (the product's residual epilogue), or, when recording, into
// c->mix first and then x += mix.
int mixer_out(laya_decoder* c, const QMat& w, int T, int layer, bool keep_mix) {
    const int h = c->d.hidden;
    if (!c->record && !keep_mix) return product(c, w, T, q8::EPI_RESID, c->x, h);
    RC(product(c, w, T, q8::EPI_STORE, c->mix, h));
    RC(record_copy(c, "layers." + std::to_string(layer) + ".mixer", c->mix, static_cast<size_t>(T) * h));
    return dec_add(c->x, c->mix, static_cast<size_t>(T) * h, c->stream);
}

// LinearAttention (Qwen35Model.cs:784-921).
int linear_mixer(laya_decoder* c, const Layer& L, int T, int n_seq, int layer, bool keep_mix) {
    const laya_decoder_desc& d = c->d;
    RC(rms_codes(c, L.in_norm, T));
    RC(product(c, L.mix_in, T, q8::EPI_STORE, c->big, c->ld_in));
    dec::ConvArgs cv{};
    cv.T = T; cv.cd = c->cd; cv.K = d.conv_kernel; cv.in = c->big; cv.ld_in = c->ld_in; cv.w = L.conv_w;
    cv.tok_seq = c->tok_seq; cv.seq_start = c->seq_start; cv.out = c->conv;
    cv.tails = c->with_states ? seq_table<float>(c, layer, 0) : nullptr;
    RC(dec_conv_silu(cv, c->stream));
    if (c->with_states) {
        dec::ConvStateArgs cs{};
        cs.n_seq = n_seq; cs.cd = c->cd; cs.K = d.conv_kernel; cs.in = c->big; cs.ld_in = c->ld_in;
        cs.seq_start = c->seq_start; cs.seq_len = c->seq_len; cs.tails = cv.tails;
        if (c->cur_snaps) { cs.snap_begin = c->snap_begin; cs.snap_at = c->snap_at; cs.snap_tails = snap_table<float>(c, layer, 0); }
        RC(dec_conv_state(cs, c->stream));
    }
    dec::HeadsArgs hd{};
    hd.T = T; hd.kh = d.lin_k_heads; hd.vh = d.lin_v_heads; hd.dk = d.lin_k_dim; hd.key_dim = c->key_dim; hd.cd = c->cd;
    hd.conv = c->conv; hd.qscale = 1.0f / static_cast<float>(std::sqrt(static_cast<double>(d.lin_k_dim)));
    hd.proj = c->big; hd.ld_proj = c->ld_in; hd.b_col = c->cd + c->vd; hd.a_col = c->cd + c->vd + d.lin_v_heads;
    hd.dt_bias = L.dt_bias; hd.neg_a = L.neg_a; hd.beta = c->beta; hd.decay = c->decay;
    RC(dec_deltanet_heads(hd, c->stream));
    dec::DeltaArgs dr{};
    dr.dk = d.lin_k_dim; dr.dv = d.lin_v_dim; dr.vh = d.lin_v_heads; dr.ratio = d.lin_v_heads / d.lin_k_heads;
    dr.key_dim = c->key_dim; dr.cd = c->cd; dr.conv = c->conv; dr.beta = c->beta; dr.decay = c->decay;
    dr.seq_start = c->seq_start; dr.seq_len = c->seq_len; dr.out = c->core; dr.ld_out = c->vd;
    dr.err = c->err;
    dr.chunked = c->chunked_rule && !c->with_states;
    if (c->with_states) {
        dr.rec = seq_table<float>(c, layer, 1);
        if (c->cur_snaps) { dr.snap_begin = c->snap_begin; dr.snap_at = c->snap_at; dr.snap_rec = snap_table<float>(c, layer, 1); }
    }
    const double rule_ops = static_cast<double>(T) * d.lin_v_heads * d.lin_k_dim * d.lin_v_dim * 8.0;
    RC(timed(c, 1, rule_ops, [&] { return dec_delta_rule(dr, n_seq, c->stream); }));
    RC(record_copy(c, "layers." + std::to_string(layer) + ".rule", c->core, static_cast<size_t>(T) * c->vd));
    dec::GatedArgs gn{};
    gn.T = T; gn.vh = d.lin_v_heads; gn.dv = d.lin_v_dim; gn.core = c->core; gn.ld_core = c->vd;
    gn.z = c->big + c->cd; gn.ld_z = c->ld_in; gn.weight = L.gnorm; gn.eps = d.eps; gn.out = c->core; gn.ld_out = c->vd;
    RC(dec_gated_norm(gn, c->stream));
    RC(q8::quantize_activations(c->core, T, c->vd, c->vd, c->qa, c->da, c->ldx, c->stream));
    return mixer_out(c, L.mix_out, T, layer, keep_mix);
}

// FullAttention (Qwen35Model.cs:628-731).
int full_mixer(laya_decoder* c, const Layer& L, int T, long long pairs, int layer, bool keep_mix) {
    const laya_decoder_desc& d = c->d;
    RC(rms_codes(c, L.in_norm, T));
    RC(product(c, L.mix_in, T, q8::EPI_STORE, c->big, c->nqkv));
    dec::PrepArgs pp{};
    pp.T = T; pp.heads = d.heads; pp.kv_heads = d.kv_heads; pp.hd = d.head_dim; pp.half = c->half;
    pp.q_width = c->q_width; pp.qkv = c->big; pp.ld_qkv = c->nqkv; pp.qnorm = L.qnorm; pp.knorm = L.knorm;
    pp.eps = d.eps; pp.cosv = c->cosv; pp.sinv = c->sinv; pp.tok_seq = c->tok_seq; pp.seq_start = c->seq_start;
    pp.pos0 = c->pos0; pp.q16 = c->q16; pp.kc = seq_table<__half>(c, layer, 0); pp.vc = seq_table<__half>(c, layer, 1);
    dec::AttnArgs at{};
    at.heads = d.heads; at.kv_heads = d.kv_heads; at.q16 = c->q16; at.kc = pp.kc; at.vc = pp.vc;
    at.tile_seq = c->tile_seq; at.tile_p0 = c->tile_p0; at.seq_start = c->seq_start; at.seq_len = c->seq_len;
    at.pos0 = c->pos0;
    at.scale = 1.0f / static_cast<float>(std::sqrt(static_cast<double>(d.head_dim)));
    at.qkv = c->big; at.ld_qkv = c->nqkv; at.out = c->core; at.ld_out = d.heads * d.head_dim;
    at.err = c->err;
    const double att_ops = 4.0 * static_cast<double>(pairs) * d.heads * d.head_dim;
    RC(timed(c, 2, att_ops, [&] {
        int rc = dec_attn_prep(pp, c->stream);
        return rc != OK ? rc : dec_attention(at, c->n_tiles, d.head_dim, c->stream);
    }));
    RC(q8::quantize_activations(c->core, T, d.heads * d.head_dim, d.heads * d.head_dim, c->qa, c->da, c->ldx, c->stream));
    return mixer_out(c, L.mix_out, T, layer, keep_mix);
}

// Mlp (Qwen35Model.cs:602-621): the [gate | up] product's epilogue applies silu(gate) · up and quantizes it for the
// down projection (the rows of gate_up are stored in [32 gate | 32 up] groups).
int mlp(laya_decoder* c, const Layer& L, int T, float* x = nullptr) {
    x = x ? x : c->x;
    RC(rms_codes(c, L.post_norm, T, x));
    q8::GemmArgs a{};
    a.M = T; a.N = L.gate_up.N; a.K = L.gate_up.K;
    a.qx = c->qa; a.dx = c->da; a.ldx = c->ldx;
    a.qw = L.gate_up.q; a.dw = L.gate_up.d; a.ldw = L.gate_up.ldw;
    a.epi = q8::EPI_SWIGLU_Q8;
    a.qout = c->qa2; a.ldqo = c->d.intermediate; a.qsc = c->da2; a.ldqs = c->ldx;
    a.err = c->err;
    RC(timed(c, 0, 2.0 * T * static_cast<double>(a.N) * a.K, [&] { return q8::gemm(a, c->stream); }));
    return product_from(c, L.down, T, q8::EPI_RESID, x, c->d.hidden, c->qa2, c->da2);
}

int run_layer(laya_decoder* c, int i, int T, int n_seq, long long pairs, bool keep_mix) {
    const Layer& L = c->layers[i];
    if (L.kind == LAYA_DECODER_FULL) RC(full_mixer(c, L, T, pairs, i, keep_mix));
    else RC(linear_mixer(c, L, T, n_seq, i, keep_mix));
    RC(mlp(c, L, T));
    return record_copy(c, "layers." + std::to_string(i), c->x, static_cast<size_t>(T) * c->d.hidden);
}

// The last layer when it is full attention and nothing is recorded (Qwen35Model.cs:488-490, ReadoutRows :563-573):
// every row's keys and values are made (later reads attend to them), but only the tiles holding each sequence's last
// row go through attention, and only those rows through o_proj and the MLP — gathered into xl, where the final norm
// reads them.  Rows are independent in every product, so the readout is the unpruned forward's, bit for bit.
int last_layer_pruned(laya_decoder* c, const Layer& L, int T, int n_seq) {
    const laya_decoder_desc& d = c->d;
    const int h = d.hidden, ao = d.heads * d.head_dim;
    RC(rms_codes(c, L.in_norm, T));
    RC(product(c, L.mix_in, T, q8::EPI_STORE, c->big, c->nqkv));
    dec::PrepArgs pp{};
    pp.T = T; pp.heads = d.heads; pp.kv_heads = d.kv_heads; pp.hd = d.head_dim; pp.half = c->half;
    pp.q_width = c->q_width; pp.qkv = c->big; pp.ld_qkv = c->nqkv; pp.qnorm = L.qnorm; pp.knorm = L.knorm;
    pp.eps = d.eps; pp.cosv = c->cosv; pp.sinv = c->sinv; pp.tok_seq = c->tok_seq; pp.seq_start = c->seq_start;
    const int layer = d.layers - 1;
    pp.pos0 = c->pos0; pp.q16 = c->q16; pp.kc = seq_table<__half>(c, layer, 0); pp.vc = seq_table<__half>(c, layer, 1);
    dec::AttnArgs at{};
    at.heads = d.heads; at.kv_heads = d.kv_heads; at.q16 = c->q16; at.kc = pp.kc; at.vc = pp.vc;
    at.tile_seq = c->lt_seq; at.tile_p0 = c->lt_p0; at.seq_start = c->seq_start; at.seq_len = c->seq_len;
    at.pos0 = c->pos0;
    at.scale = 1.0f / static_cast<float>(std::sqrt(static_cast<double>(d.head_dim)));
    at.qkv = c->big; at.ld_qkv = c->nqkv; at.out = c->core; at.ld_out = ao;
    at.err = c->err;
    RC(dec_attn_prep(pp, c->stream));
    RC(dec_attention(at, n_seq, d.head_dim, c->stream));
    RC(dec_gather_rows(c->core, ao, c->last_row, n_seq, ao, c->corel, ao, c->stream));
    RC(dec_gather_rows(c->x, h, c->last_row, n_seq, h, c->xl, h, c->stream));
    RC(q8::quantize_activations(c->corel, n_seq, ao, ao, c->qa, c->da, c->ldx, c->stream));
    RC(product(c, L.mix_out, n_seq, q8::EPI_RESID, c->xl, h));
    return mlp(c, L, n_seq, c->xl);
}

// The states a forward's sequences continue, and the snapshot states its checkpoints fill (validated by the caller).
struct StateView {
    laya_decoder_state* const* states = nullptr;   // [n_seq]
    const int32_t* n_cp = nullptr;                 // [n_seq] or null
    const int32_t* cps = nullptr;                  // concatenated checkpoints
    laya_decoder_state* const* snaps = nullptr;    // [n_snap]
    int n_snap = 0;
};

// Host metadata of one forward → pinned staging → one copy.  Returns the causal (query, key) pairs of full attention.
int stage(laya_decoder* c, const int32_t* ids_host, const int32_t* seq_len, int n_seq, const int32_t* labels,
          int n_labels, int* T_out, long long* pairs_out, const StateView* sv = nullptr) {
    if (n_seq <= 0 || n_seq > c->d.max_seqs) { set_error("sequence count outside 1..max_seqs"); return ERR_ARGUMENT; }
    long long T = 0, pairs = 0;
    int tiles = 0;
    for (int s = 0; s < n_seq; ++s) {
        if (seq_len[s] <= 0) { set_error("every sequence needs at least one token"); return ERR_ARGUMENT; }
        const long long p0 = sv ? sv->states[s]->length : 0;
        T += seq_len[s];
        pairs += static_cast<long long>(seq_len[s]) * (seq_len[s] + 1) / 2 + p0 * seq_len[s];
        tiles += (seq_len[s] + 63) / 64;
    }
    if (T > c->d.max_tokens) { set_error("more tokens than max_tokens"); return ERR_ARGUMENT; }
    if (n_labels < 0 || (n_labels > 0 && !labels)) { set_error("invalid label list"); return ERR_ARGUMENT; }
    for (int l = 0; l < n_labels; ++l)
        if (labels[l] < 0 || labels[l] >= c->d.vocab) { set_error("label id outside the vocabulary"); return ERR_OUT_OF_RANGE; }
    const int n_snap = sv ? sv->n_snap : 0;
    const size_t n_ptr = 2 * static_cast<size_t>(c->d.layers) * (n_seq + n_snap);
    const size_t need = static_cast<size_t>(ids_host ? T : 0) + T + 3 * static_cast<size_t>(n_seq) + 2 * tiles +
                        n_labels + n_seq + (n_seq + 1) + n_snap + 2 * n_seq + 1 + 2 * n_ptr;
    if (c->in_pending) { LAYA_CUDA(cudaEventSynchronize(c->in_done)); c->in_pending = false; }
    if (need > c->in_cap) {
        if (c->in_host) cudaFreeHost(c->in_host);
        if (c->in_dev) cudaFree(c->in_dev);
        c->in_host = nullptr; c->in_dev = nullptr;
        c->in_cap = need + 1024;
        LAYA_CUDA(cudaMallocHost(&c->in_host, c->in_cap * sizeof(int32_t)));
        LAYA_CUDA(cudaMalloc(&c->in_dev, c->in_cap * sizeof(int32_t)));
    }
    int32_t* h = c->in_host;
    size_t o = 0;
    auto slot = [&](size_t n, int32_t** dev) {
        *dev = c->in_dev + o;
        int32_t* p = h + o;
        o += n;
        return p;
    };
    int32_t* ids_dev = nullptr;
    if (ids_host) memcpy(slot(T, &ids_dev), ids_host, sizeof(int32_t) * T);
    int32_t* ts = slot(T, &c->tok_seq);
    int32_t* ss = slot(n_seq, &c->seq_start);
    int32_t* sl = slot(n_seq, &c->seq_len);
    int32_t* lr = slot(n_seq, &c->last_row);
    int32_t* tsq = slot(tiles, &c->tile_seq);
    int32_t* tp0 = slot(tiles, &c->tile_p0);
    int32_t* lb = slot(n_labels, &c->labels);
    int32_t* ps = slot(n_seq, &c->pos0);
    int32_t* sb = slot(n_seq + 1, &c->snap_begin);
    int32_t* sa = slot(n_snap, &c->snap_at);
    int32_t* lts = slot(n_seq, &c->lt_seq);
    int32_t* ltp = slot(n_seq, &c->lt_p0);
    if (o & 1) ++o;   // 8-byte alignment of the pointer tables (the device buffer is 256-byte aligned)
    int32_t* dummy = nullptr;
    uint64_t* pt = reinterpret_cast<uint64_t*>(slot(2 * n_ptr, &dummy));
    c->ptrs = reinterpret_cast<uint64_t*>(dummy);
    int start = 0;
    std::vector<std::pair<int, int>> tl;   // (key positions before the tile's last query, tile index)
    std::vector<std::pair<int, int>> tile_of;
    for (int s = 0; s < n_seq; ++s) {
        ss[s] = start; sl[s] = seq_len[s]; lr[s] = start + seq_len[s] - 1;
        ps[s] = sv ? sv->states[s]->length : 0;
        lts[s] = s;
        ltp[s] = (seq_len[s] - 1) / 64 * 64;
        for (int t = 0; t < seq_len[s]; ++t) ts[start + t] = s;
        for (int p0 = 0; p0 < seq_len[s]; p0 += 64) {
            tl.push_back({ps[s] + p0, static_cast<int>(tile_of.size())});
            tile_of.push_back({p0, s});
        }
        start += seq_len[s];
    }
    // longest causal rows first
    std::stable_sort(tl.begin(), tl.end(), [](const std::pair<int, int>& a, const std::pair<int, int>& b) { return a.first > b.first; });
    for (int i = 0; i < tiles; ++i) { tsq[i] = tile_of[tl[i].second].second; tp0[i] = tile_of[tl[i].second].first; }
    sb[0] = 0;
    for (int s = 0; s < n_seq; ++s) {
        const int n = (sv && sv->n_cp) ? sv->n_cp[s] : 0;
        for (int k = 0; k < n; ++k) sa[sb[s] + k] = sv->cps[sb[s] + k];
        sb[s + 1] = sb[s] + n;
    }
    const size_t ldkv = static_cast<size_t>(c->d.kv_heads) * c->d.head_dim;
    for (int i = 0; i < c->d.layers; ++i) {
        const bool full = c->kinds[i] == LAYA_DECODER_FULL;
        uint64_t* a = pt + (2 * static_cast<size_t>(i)) * n_seq;
        uint64_t* b = a + n_seq;
        for (int s = 0; s < n_seq; ++s) {
            if (sv) {
                const laya_decoder_state* st = sv->states[s];
                a[s] = reinterpret_cast<uint64_t>(full ? static_cast<void*>(st->k[i]) : static_cast<void*>(st->tail[i]));
                b[s] = reinterpret_cast<uint64_t>(full ? static_cast<void*>(st->v[i]) : static_cast<void*>(st->rec[i]));
            } else {
                a[s] = full ? reinterpret_cast<uint64_t>(c->k16 + ss[s] * ldkv) : 0;
                b[s] = full ? reinterpret_cast<uint64_t>(c->v16 + ss[s] * ldkv) : 0;
            }
        }
        uint64_t* sa_ = pt + 2 * static_cast<size_t>(c->d.layers) * n_seq + (2 * static_cast<size_t>(i)) * n_snap;
        for (int k = 0; k < n_snap; ++k) {
            const laya_decoder_state* st = sv->snaps[k];
            sa_[k] = full ? 0 : reinterpret_cast<uint64_t>(st->tail[i]);
            sa_[n_snap + k] = full ? 0 : reinterpret_cast<uint64_t>(st->rec[i]);
        }
    }
    c->cur_seqs = n_seq;
    c->cur_snaps = n_snap;
    c->with_states = sv != nullptr;
    if (n_labels) memcpy(lb, labels, sizeof(int32_t) * n_labels);
    c->n_tiles = tiles;
    LAYA_CUDA(cudaMemcpyAsync(c->in_dev, h, o * sizeof(int32_t), cudaMemcpyHostToDevice, c->stream));
    LAYA_CUDA(cudaEventRecord(c->in_done, c->stream));
    c->in_pending = true;
    if (ids_host) c->ids = ids_dev;
    *T_out = static_cast<int>(T);
    *pairs_out = pairs;
    return OK;
}

int ready(laya_decoder* c) {
    if (c->have.size() == c->parts.size() + c->vecs.size()) return OK;
    for (auto& p : c->parts)
        if (!c->have.count(p.first)) { set_error("missing tensor " + p.first); return ERR_NOT_FOUND; }
    for (auto& v : c->vecs)
        if (!c->have.count(v.first)) { set_error("missing tensor " + v.first); return ERR_NOT_FOUND; }
    return OK;
}

// Embeddings → layers → final norm of every sequence's last row → label logits.
int forward_body(laya_decoder* c, int T, int n_seq, long long pairs, int n_labels, float* hidden, float* logits) {
    const int h = c->d.hidden;
    RC(dec_embed(c->ids, T, h, c->d.vocab, c->table.q, c->table.d, c->table.ldw, c->x, c->err, c->stream));
    RC(record_copy(c, "embeddings", c->x, static_cast<size_t>(T) * h));
    const bool prune = !c->record && c->layers.back().kind == LAYA_DECODER_FULL;
    for (int i = 0; i < c->d.layers - (prune ? 1 : 0); ++i) RC(run_layer(c, i, T, n_seq, pairs, false));
    if (prune) RC(last_layer_pruned(c, c->layers.back(), T, n_seq));
    dec::RmsArgs r{};
    r.rows = n_seq; r.n = h; r.x = prune ? c->xl : c->x; r.row_map = prune ? nullptr : c->last_row;
    r.scale = c->final_norm; r.eps = c->d.eps;
    r.out32 = hidden ? hidden : c->hid; r.q = c->qlast; r.d = c->dlast; r.ldd = c->ldl;
    RC(dec_rms_q8(r, c->stream));
    if (c->record) {
        dec::RmsArgs a = r;
        a.rows = T; a.row_map = nullptr; a.out32 = c->mix; a.q = nullptr;
        RC(dec_rms_q8(a, c->stream));
        RC(record_copy(c, "norm", c->mix, static_cast<size_t>(T) * h));
    }
    if (n_labels > 0 && logits) {
        dec::LogitArgs lg{};
        lg.n_seq = n_seq; lg.n_labels = n_labels; lg.n = h; lg.vocab = c->d.vocab;
        lg.qx = c->qlast; lg.dx = c->dlast; lg.ldx = c->ldl;
        lg.qw = c->table.q; lg.dw = c->table.d; lg.ldw = c->table.ldw;
        lg.labels = c->labels; lg.logits = logits; lg.err = c->err;
        RC(dec_q8_logits(lg, c->stream));
    }
    return OK;
}

int ensure_logits(laya_decoder* c, size_t n) {
    if (static_cast<size_t>(c->logit_cap) >= n) return OK;
    if (c->logit_buf) cudaFree(c->logit_buf);
    c->logit_buf = nullptr;
    LAYA_CUDA(cudaMalloc(&c->logit_buf, std::max<size_t>(n, 64) * sizeof(float)));
    c->logit_cap = static_cast<int>(std::max<size_t>(n, 64));
    return OK;
}

std::string strip(const char* name) {
    std::string n(name);
    for (const char* p : {"model.language_model.", "model."})
        if (n.rfind(p, 0) == 0) return n.substr(strlen(p));
    return n;
}

// Register the tensors of the checkpoint: stacked projection parts and vectors.
void register_tensors(laya_decoder* c) {
    const laya_decoder_desc& d = c->d;
    c->parts["embed_tokens.weight"] = {&c->table, 0, d.vocab};
    c->vecs["norm.weight"] = {&c->final_norm, d.hidden, V_ONE_PLUS};
    for (int i = 0; i < d.layers; ++i) {
        Layer& L = c->layers[i];
        const std::string p = "layers." + std::to_string(i) + ".";
        c->vecs[p + "input_layernorm.weight"] = {&L.in_norm, d.hidden, V_ONE_PLUS};
        c->vecs[p + "post_attention_layernorm.weight"] = {&L.post_norm, d.hidden, V_ONE_PLUS};
        c->parts[p + "mlp.gate_proj.weight"] = {&L.gate_up, 0, d.intermediate, true};
        c->parts[p + "mlp.up_proj.weight"] = {&L.gate_up, 32, d.intermediate, true};
        c->parts[p + "mlp.down_proj.weight"] = {&L.down, 0, d.hidden};
        if (L.kind == LAYA_DECODER_FULL) {
            const std::string a = p + "self_attn.";
            const int kvw = d.kv_heads * d.head_dim;
            c->parts[a + "q_proj.weight"] = {&L.mix_in, 0, c->q_width};
            c->parts[a + "k_proj.weight"] = {&L.mix_in, c->q_width, kvw};
            c->parts[a + "v_proj.weight"] = {&L.mix_in, c->q_width + kvw, kvw};
            c->parts[a + "o_proj.weight"] = {&L.mix_out, 0, d.hidden};
            c->vecs[a + "q_norm.weight"] = {&L.qnorm, d.head_dim, V_ONE_PLUS};
            c->vecs[a + "k_norm.weight"] = {&L.knorm, d.head_dim, V_ONE_PLUS};
        } else {
            const std::string a = p + "linear_attn.";
            c->parts[a + "in_proj_qkv.weight"] = {&L.mix_in, 0, c->cd};
            c->parts[a + "in_proj_z.weight"] = {&L.mix_in, c->cd, c->vd};
            c->parts[a + "in_proj_b.weight"] = {&L.mix_in, c->cd + c->vd, d.lin_v_heads};
            c->parts[a + "in_proj_a.weight"] = {&L.mix_in, c->cd + c->vd + d.lin_v_heads, d.lin_v_heads};
            c->parts[a + "out_proj.weight"] = {&L.mix_out, 0, d.hidden};
            c->vecs[a + "conv1d.weight"] = {&L.conv_w, static_cast<int64_t>(c->cd) * d.conv_kernel, V_CONV};
            c->vecs[a + "A_log"] = {&L.neg_a, d.lin_v_heads, V_NEG_EXP};
            c->vecs[a + "dt_bias"] = {&L.dt_bias, d.lin_v_heads, V_PLAIN};
            c->vecs[a + "norm.weight"] = {&L.gnorm, d.lin_v_dim, V_PLAIN};
        }
    }
}

int check_desc(const laya_decoder_desc& d) {
    auto bad = [](const char* m) { set_error(m); return ERR_ARGUMENT; };
    if (d.hidden <= 0 || d.hidden % 32 || d.intermediate <= 0 || d.intermediate % 32 || d.layers < 0 || d.vocab <= 0)
        return bad("hidden and intermediate must be positive multiples of 32");
    if (d.layers > 0 && !d.layer_kinds) return bad("layer_kinds is required");
    if (d.heads <= 0 || d.kv_heads <= 0 || d.heads % d.kv_heads) return bad("kv_heads must divide heads");
    if (d.head_dim != 32 && d.head_dim != 64 && d.head_dim != 128) return bad("head_dim must be 32, 64 or 128");
    if (d.rotary_dim < 0 || d.rotary_dim > d.head_dim || d.rotary_dim % 2) return bad("rotary_dim must be even and at most head_dim");
    if (d.lin_k_heads <= 0 || d.lin_v_heads <= 0 || d.lin_v_heads % d.lin_k_heads) return bad("lin_v_heads must be a multiple of lin_k_heads");
    if (d.lin_k_dim != 16 && d.lin_k_dim != 32 && d.lin_k_dim != 64 && d.lin_k_dim != 128) return bad("lin_k_dim must be 16, 32, 64 or 128");
    if (d.lin_v_dim <= 0 || d.lin_v_dim > 128) return bad("lin_v_dim must be 1..128");
    if ((d.lin_v_heads * d.lin_v_dim) % 32 || (d.heads * d.head_dim) % 32) return bad("value and attention widths must be multiples of 32");
    if (d.conv_kernel <= 0 || d.conv_kernel > 16) return bad("conv_kernel must be 1..16");
    if (d.max_tokens <= 0 || d.max_seqs <= 0) return bad("max_tokens and max_seqs must be positive");
    if (!(d.eps > 0.0f)) return bad("eps must be positive");
    for (int i = 0; i < d.layers; ++i)
        if (d.layer_kinds[i] != LAYA_DECODER_LINEAR && d.layer_kinds[i] != LAYA_DECODER_FULL) return bad("unknown layer kind");
    return OK;
}

// A stream-ordered block from the decoder's pool.
cudaError_t pool_alloc(laya_decoder* c, void** p, size_t bytes) { return cudaMallocFromPoolAsync(p, bytes, c->pool, c->stream); }

// RoPE tables for positions [0, positions) (Qwen35Model.cs:247-253): inv_freq = 1/θ^(2i/rotary_dim) and
// angle = pos·inv_freq in fp32.  Grown (rebuilt) when a state reads past them; the old tables are freed after the work
// queued on the stream.
int ensure_rope(laya_decoder* c, int positions) {
    if (positions <= c->rope_cap) return OK;
    const laya_decoder_desc& d = c->d;
    const int hf = std::max(c->half, 1);
    const size_t n = static_cast<size_t>(positions) * hf;
    std::vector<float> cs(n), sn(n), inv(hf);
    for (int i = 0; i < c->half; ++i)
        inv[i] = 1.0f / std::pow(static_cast<float>(d.rope_theta), static_cast<float>(2 * i) / static_cast<float>(d.rotary_dim));
    for (size_t p = 0; p < static_cast<size_t>(positions); ++p)
        for (int i = 0; i < c->half; ++i) {
            const float ang = static_cast<float>(p) * inv[i];
            cs[p * hf + i] = static_cast<float>(std::cos(static_cast<double>(ang)));
            sn[p * hf + i] = static_cast<float>(std::sin(static_cast<double>(ang)));
        }
    float *nc = nullptr, *ns = nullptr;
    LAYA_CUDA(cudaMallocAsync(&nc, n * sizeof(float), c->stream));
    cudaError_t e = cudaMallocAsync(&ns, n * sizeof(float), c->stream);
    if (e != cudaSuccess) { cudaFreeAsync(nc, c->stream); return cuda_fail(e, "cudaMallocAsync"); }
    LAYA_CUDA(cudaMemcpyAsync(nc, cs.data(), n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    LAYA_CUDA(cudaMemcpyAsync(ns, sn.data(), n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));   // the host tables go out of scope
    if (c->cosv) cudaFreeAsync(c->cosv, c->stream);
    if (c->sinv) cudaFreeAsync(c->sinv, c->stream);
    c->cosv = nc;
    c->sinv = ns;
    c->rope_cap = positions;
    return OK;
}

int create(laya_decoder* c) {
    const laya_decoder_desc& d = c->d;
    c->key_dim = d.lin_k_heads * d.lin_k_dim;
    c->vd = d.lin_v_heads * d.lin_v_dim;
    c->cd = 2 * c->key_dim + c->vd;
    c->nin = c->cd + c->vd + 2 * d.lin_v_heads;
    c->ld_in = rup(c->nin, 4);
    c->q_width = 2 * d.heads * d.head_dim;
    c->nqkv = c->q_width + 2 * d.kv_heads * d.head_dim;
    c->half = d.rotary_dim / 2;
    c->maxK = std::max({d.hidden, d.intermediate, c->vd, d.heads * d.head_dim});
    c->ldx = rup(d.max_tokens, 128);
    c->widest = std::max(c->ld_in, c->nqkv);
    c->core_w = std::max(c->vd, d.heads * d.head_dim);
    c->ldl = rup(d.max_seqs, 4);
    const size_t T = d.max_tokens;
    LAYA_CUDA(cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking));
    c->stream = c->own;
    LAYA_CUDA(cudaEventCreateWithFlags(&c->in_done, cudaEventDisableTiming));
    RC(dalloc_t(c, &c->err, 1));
    LAYA_CUDA(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream));
    {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = c->device;
        LAYA_CUDA(cudaMemPoolCreate(&c->pool, &props));
        uint64_t keep = UINT64_MAX;   // never trim: a request's clones reuse the blocks the previous one freed
        LAYA_CUDA(cudaMemPoolSetAttribute(c->pool, cudaMemPoolAttrReleaseThreshold, &keep));
    }

    c->layers.resize(d.layers);
    RC(alloc_qmat(c, c->table, d.vocab, d.hidden));
    bool any_full = false, any_linear = false;
    for (int i = 0; i < d.layers; ++i) {
        Layer& L = c->layers[i];
        L.kind = c->kinds[i];
        if (L.kind == LAYA_DECODER_FULL) {
            any_full = true;
            RC(alloc_qmat(c, L.mix_in, c->nqkv, d.hidden));
            RC(alloc_qmat(c, L.mix_out, d.hidden, d.heads * d.head_dim));
        } else {
            any_linear = true;
            RC(alloc_qmat(c, L.mix_in, c->nin, d.hidden));
            RC(alloc_qmat(c, L.mix_out, d.hidden, c->vd));
        }
        RC(alloc_qmat(c, L.gate_up, 2 * d.intermediate, d.hidden));
        RC(alloc_qmat(c, L.down, d.hidden, d.intermediate));
    }
    register_tensors(c);
    for (auto& v : c->vecs) RC(dalloc_t(c, v.second.dst, static_cast<size_t>(v.second.count)));

    RC(dalloc_t(c, &c->x, T * d.hidden));
    RC(dalloc_t(c, &c->mix, T * d.hidden));
    RC(dalloc_t(c, &c->big, T * c->widest));
    RC(dalloc_t(c, &c->core, T * c->core_w));
    RC(dalloc_t(c, &c->qa, T * c->maxK));
    RC(dalloc_t(c, &c->da, static_cast<size_t>(c->maxK / 32) * c->ldx));
    RC(dalloc_t(c, &c->qa2, T * d.intermediate));
    RC(dalloc_t(c, &c->da2, static_cast<size_t>(d.intermediate / 32) * c->ldx));
    if (any_linear) {
        RC(dalloc_t(c, &c->conv, T * c->cd));
        RC(dalloc_t(c, &c->beta, T * d.lin_v_heads));
        RC(dalloc_t(c, &c->decay, T * d.lin_v_heads));
    }
    if (any_full) {
        RC(dalloc_t(c, &c->q16, T * d.heads * d.head_dim));
        RC(dalloc_t(c, &c->k16, T * d.kv_heads * d.head_dim));
        RC(dalloc_t(c, &c->v16, T * d.kv_heads * d.head_dim));
        RC(ensure_rope(c, static_cast<int>(T)));
        RC(dalloc_t(c, &c->xl, static_cast<size_t>(d.max_seqs) * d.hidden));
        RC(dalloc_t(c, &c->corel, static_cast<size_t>(d.max_seqs) * d.heads * d.head_dim));
    }
    RC(dalloc_t(c, &c->hid, static_cast<size_t>(d.max_seqs) * d.hidden));
    RC(dalloc_t(c, &c->qlast, static_cast<size_t>(d.max_seqs) * d.hidden));
    RC(dalloc_t(c, &c->dlast, static_cast<size_t>(d.hidden / 32) * c->ldl));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    return OK;
}

// Copies a part's codes q [rows, K] and scales d [K/32, rows] (device) into its rows of the stacked matrix.
int place(laya_decoder* c, const Part& p, const q8::code_t* q, const float* d) {
    QMat& m = *p.m;
    const size_t K = m.K, nb = m.K / 32;
    if (!p.interleaved) {
        LAYA_CUDA(cudaMemcpyAsync(m.q + static_cast<size_t>(p.row0) * K, q, sizeof(q8::code_t) * p.rows * K,
                                  cudaMemcpyDeviceToDevice, c->stream));
        LAYA_CUDA(cudaMemcpy2DAsync(m.d + p.row0, sizeof(float) * m.ldw, d, sizeof(float) * p.rows,
                                    sizeof(float) * p.rows, nb, cudaMemcpyDeviceToDevice, c->stream));
        return OK;
    }
    const int groups = p.rows / 32;
    LAYA_CUDA(cudaMemcpy2DAsync(m.q + static_cast<size_t>(p.row0) * K, sizeof(q8::code_t) * 64 * K, q,
                                sizeof(q8::code_t) * 32 * K, sizeof(q8::code_t) * 32 * K, groups,
                                cudaMemcpyDeviceToDevice, c->stream));
    for (size_t b = 0; b < nb; ++b)
        LAYA_CUDA(cudaMemcpy2DAsync(m.d + b * m.ldw + p.row0, sizeof(float) * 64, d + b * p.rows, sizeof(float) * 32,
                                    sizeof(float) * 32, groups, cudaMemcpyDeviceToDevice, c->stream));
    return OK;
}

struct Scratch {   // temporaries of one upload, freed on every path
    std::vector<void*> p;
    ~Scratch() {
        for (void* x : p) cudaFree(x);
    }
    template <class T>
    int get(T** out, size_t count) {
        void* x = nullptr;
        cudaError_t e = cudaMalloc(&x, std::max<size_t>(count * sizeof(T), 16));
        if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
        p.push_back(x);
        *out = static_cast<T*>(x);
        return OK;
    }
};

// Quantize a part from fp32 host rows on the device (Q8_0.QuantizeWeightBlock), then place it.
int fill_rows(laya_decoder* c, const Part& p, const float* host) {
    const size_t K = p.m->K, n = static_cast<size_t>(p.rows) * K;
    Scratch t;
    float *w = nullptr, *d = nullptr;
    q8::code_t* q = nullptr;
    RC(t.get(&w, n));
    RC(t.get(&q, n));
    RC(t.get(&d, n / 32));
    LAYA_CUDA(cudaMemcpyAsync(w, host, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    RC(q8::quantize_weights(w, p.rows, static_cast<int>(K), q, d, p.rows, c->stream));
    RC(place(c, p, q, d));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    return OK;
}

// A part already in Q8_0: int8 codes [rows, K] and fp16 scales [rows, K/32] from the host.
int fill_rows_q8(laya_decoder* c, const Part& p, const int8_t* q_host, const uint16_t* d_fp16) {
    const int nb = p.m->K / 32;
    const size_t n = static_cast<size_t>(p.rows) * p.m->K;
    std::vector<float> dt(static_cast<size_t>(nb) * p.rows);
    for (int r = 0; r < p.rows; ++r)
        for (int b = 0; b < nb; ++b) dt[static_cast<size_t>(b) * p.rows + r] = half_bits(d_fp16[static_cast<size_t>(r) * nb + b]);
    Scratch t;
    int8_t* q8 = nullptr;
    q8::code_t* q = nullptr;
    float* d = nullptr;
    RC(t.get(&q8, n));
    RC(t.get(&q, n));
    RC(t.get(&d, dt.size()));
    LAYA_CUDA(cudaMemcpyAsync(q8, q_host, n, cudaMemcpyHostToDevice, c->stream));
    LAYA_CUDA(cudaMemcpyAsync(d, dt.data(), dt.size() * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    RC(q8::widen_codes(q8, q, n, c->stream));
    RC(place(c, p, q, d));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    return OK;
}

// ------------------------------------------------------------------------------------------------ states
size_t pad256(size_t b) { return (b + 255) / 256 * 256; }
size_t state_fixed_bytes(const laya_decoder* c) {
    const laya_decoder_desc& d = c->d;
    size_t b = 0;
    for (int i = 0; i < d.layers; ++i)
        if (c->kinds[i] != LAYA_DECODER_FULL)
            b += pad256(sizeof(float) * (d.conv_kernel - 1) * c->cd) +
                 pad256(sizeof(float) * static_cast<size_t>(d.lin_v_heads) * d.lin_k_dim * d.lin_v_dim);
    return b;
}
size_t state_kv_bytes(const laya_decoder* c, int capacity) {   // one cache (keys or values) of one layer
    return pad256(sizeof(__half) * static_cast<size_t>(capacity) * c->d.kv_heads * c->d.head_dim);
}
void state_bind(laya_decoder_state* st) {
    const laya_decoder* c = st->dec;
    const laya_decoder_desc& d = c->d;
    st->tail.assign(d.layers, nullptr);
    st->rec.assign(d.layers, nullptr);
    st->k.assign(d.layers, nullptr);
    st->v.assign(d.layers, nullptr);
    char* p = st->block;
    for (int i = 0; i < d.layers; ++i)
        if (c->kinds[i] != LAYA_DECODER_FULL) {
            st->tail[i] = reinterpret_cast<float*>(p);
            p += pad256(sizeof(float) * (d.conv_kernel - 1) * c->cd);
            st->rec[i] = reinterpret_cast<float*>(p);
            p += pad256(sizeof(float) * static_cast<size_t>(d.lin_v_heads) * d.lin_k_dim * d.lin_v_dim);
        }
    const size_t kv = state_kv_bytes(c, st->capacity);
    for (int i = 0; i < d.layers; ++i)
        if (c->kinds[i] == LAYA_DECODER_FULL) {
            st->k[i] = reinterpret_cast<__half*>(p);
            p += kv;
            st->v[i] = reinterpret_cast<__half*>(p);
            p += kv;
        }
}
int n_full_layers(const laya_decoder* c) {
    int n = 0;
    for (int k : c->kinds) n += k == LAYA_DECODER_FULL;
    return n;
}
// A block for `capacity` tokens on the decoder's stream; the fixed part zeroed when `zero`.
int state_block(laya_decoder* c, int capacity, bool zero, char** block, size_t* bytes) {
    const size_t fixed = state_fixed_bytes(c);
    *bytes = std::max<size_t>(fixed + 2 * n_full_layers(c) * state_kv_bytes(c, capacity), 256);
    void* p = nullptr;
    LAYA_CUDA(pool_alloc(c, &p, *bytes));
    *block = static_cast<char*>(p);
    if (zero && fixed) LAYA_CUDA(cudaMemsetAsync(p, 0, fixed, c->stream));
    return OK;
}
// Copies what `from` holds (fixed part, keys and values of its first `from->length` positions) into `to`.
int state_copy(laya_decoder* c, const laya_decoder_state* from, laya_decoder_state* to) {
    if (from->fixed) LAYA_CUDA(cudaMemcpyAsync(to->block, from->block, from->fixed, cudaMemcpyDeviceToDevice, c->stream));
    const size_t row = sizeof(__half) * static_cast<size_t>(c->d.kv_heads) * c->d.head_dim;
    if (from->length > 0)
        for (int i = 0; i < c->d.layers; ++i)
            if (c->kinds[i] == LAYA_DECODER_FULL) {
                LAYA_CUDA(cudaMemcpyAsync(to->k[i], from->k[i], row * from->length, cudaMemcpyDeviceToDevice, c->stream));
                LAYA_CUDA(cudaMemcpyAsync(to->v[i], from->v[i], row * from->length, cudaMemcpyDeviceToDevice, c->stream));
            }
    to->length = from->length;
    return OK;
}
int state_new(laya_decoder* c, int capacity, laya_decoder_state** out) {
    laya_decoder_state* st = new laya_decoder_state();
    st->dec = c;
    st->capacity = capacity;
    st->fixed = state_fixed_bytes(c);
    const int rc = state_block(c, capacity, true, &st->block, &st->bytes);
    if (rc != OK) { delete st; return rc; }
    state_bind(st);
    c->states.insert(st);
    *out = st;
    return OK;
}
void state_free(laya_decoder_state* st) {
    if (st->dec) {
        if (st->block) cudaFreeAsync(st->block, st->dec->stream);
        st->dec->states.erase(st);
    }
    delete st;
}
// Qwen35State.GrowCache (Qwen35Model.cs:146-154): room for `needed` positions, the next power of two at least.
int state_grow(laya_decoder* c, laya_decoder_state* st, int needed) {
    if (needed <= st->capacity) return OK;
    long long cap = 1;
    while (cap < needed) cap <<= 1;
    laya_decoder_state grown;
    grown.dec = c;
    grown.capacity = static_cast<int>(std::min<long long>(cap, INT32_MAX));
    grown.fixed = st->fixed;
    RC(state_block(c, grown.capacity, false, &grown.block, &grown.bytes));
    state_bind(&grown);
    const int rc = state_copy(c, st, &grown);
    if (rc != OK) { cudaFreeAsync(grown.block, c->stream); return rc; }
    cudaFreeAsync(st->block, c->stream);
    st->block = grown.block;
    st->bytes = grown.bytes;
    st->capacity = grown.capacity;
    st->tail = grown.tail; st->rec = grown.rec; st->k = grown.k; st->v = grown.v;
    return OK;
}

int stage_input_rows(laya_decoder* c, const int32_t* seq_len, int n_seq, int* T_out, long long* pairs) {
    return stage(c, nullptr, seq_len, n_seq, nullptr, 0, T_out, pairs);
}

}  // namespace

// ================================================================================================ C ABI
extern "C" {

int laya_decoder_create(const laya_decoder_desc* desc, int device, laya_decoder** out) {
    if (!desc || !out) { set_error("null argument"); return ERR_ARGUMENT; }
    *out = nullptr;
    RC(check_desc(*desc));
    int n = 0;
    LAYA_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) { set_error("invalid device ordinal"); return ERR_ARGUMENT; }
    DeviceGuard g(device);
    laya_decoder* c = new laya_decoder();
    c->device = device;
    c->d = *desc;
    c->kinds.assign(desc->layer_kinds, desc->layer_kinds + desc->layers);
    c->d.layer_kinds = nullptr;
    const int rc = create(c);
    if (rc != OK) {
        laya_decoder_destroy(c);
        return rc;
    }
    *out = c;
    return OK;
}

int laya_decoder_destroy(laya_decoder* c) {
    if (!c) return OK;
    DeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (laya_decoder_state* st : c->states) { cudaFree(st->block); st->block = nullptr; st->dec = nullptr; }
    for (laya_decoder_mark* m : c->marks) { cudaFree(m->block); m->block = nullptr; m->dec = nullptr; }
    if (c->cosv) cudaFree(c->cosv);
    if (c->sinv) cudaFree(c->sinv);
    for (void* p : c->allocs) cudaFree(p);
    for (auto& r : c->rec) cudaFree(r.second.p);
    for (auto& e : c->ev_pool) { cudaEventDestroy(e.first); cudaEventDestroy(e.second); }
    if (c->logit_buf) cudaFree(c->logit_buf);
    if (c->in_dev) cudaFree(c->in_dev);
    if (c->in_host) cudaFreeHost(c->in_host);
    if (c->in_done) cudaEventDestroy(c->in_done);
    if (c->pool) cudaMemPoolDestroy(c->pool);
    if (c->own) cudaStreamDestroy(c->own);
    delete c;
    return OK;
}

int laya_decoder_set_stream(laya_decoder* c, void* stream) {
    if (!c) { set_error("null decoder"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    c->stream = stream ? static_cast<cudaStream_t>(stream) : c->own;
    return OK;
}

int laya_decoder_get_stream(laya_decoder* c, void** stream) {
    if (!c || !stream) { set_error("null argument"); return ERR_ARGUMENT; }
    *stream = c->stream;
    return OK;
}

int laya_decoder_synchronize(laya_decoder* c) {
    if (!c) { set_error("null decoder"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    return check_device_error(c);
}

int laya_decoder_upload(laya_decoder* c, const char* name, int dtype, const int64_t* shape, int rank, const void* host) {
    if (!c || !name || !host || rank < 0 || rank > 8 || (rank > 0 && !shape)) { set_error("invalid argument"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    const std::string n = strip(name);
    int64_t count = 1;
    for (int i = 0; i < rank; ++i) {
        if (shape[i] < 0) { set_error("negative dimension"); return ERR_ARGUMENT; }
        count *= shape[i];
    }
    std::vector<float> tmp;
    const float* src = nullptr;
    switch (dtype) {
        case LAYA_F32: src = static_cast<const float*>(host); break;
        case LAYA_BF16:
        case LAYA_F16: {
            tmp.resize(count);
            const uint16_t* b = static_cast<const uint16_t*>(host);
            for (int64_t i = 0; i < count; ++i) tmp[i] = dtype == LAYA_BF16 ? bf16_bits(b[i]) : half_bits(b[i]);
            src = tmp.data();
            break;
        }
        default: set_error("unsupported dtype for a float tensor"); return ERR_ARGUMENT;
    }
    auto pt = c->parts.find(n);
    if (pt != c->parts.end()) {
        const Part& p = pt->second;
        if (rank != 2 || shape[0] != p.rows || shape[1] != p.m->K) {
            set_error(n + ": expected [" + std::to_string(p.rows) + ", " + std::to_string(p.m->K) + "]");
            return ERR_ARGUMENT;
        }
        RC(fill_rows(c, p, src));
        c->have.insert(n);
        return OK;
    }
    auto vt = c->vecs.find(n);
    if (vt == c->vecs.end()) { set_error("no decoder tensor named " + n); return ERR_NOT_FOUND; }
    const Vec& v = vt->second;
    if (count != v.count) { set_error(n + ": expected " + std::to_string(v.count) + " values"); return ERR_ARGUMENT; }
    std::vector<float> val(count);
    switch (v.kind) {
        case V_PLAIN: memcpy(val.data(), src, count * sizeof(float)); break;
        case V_ONE_PLUS: for (int64_t i = 0; i < count; ++i) val[i] = 1.0f + src[i]; break;
        case V_NEG_EXP: for (int64_t i = 0; i < count; ++i) val[i] = -std::exp(src[i]); break;
        case V_CONV: {   // [channels, 1, taps] → [taps, channels]
            const int K = c->d.conv_kernel, cd = c->cd;
            for (int ch = 0; ch < cd; ++ch)
                for (int j = 0; j < K; ++j) val[static_cast<size_t>(j) * cd + ch] = src[static_cast<size_t>(ch) * K + j];
            break;
        }
    }
    LAYA_CUDA(cudaMemcpyAsync(*v.dst, val.data(), count * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    c->have.insert(n);
    return OK;
}

int laya_decoder_upload_q8_0(laya_decoder* c, const char* name, const int8_t* q, const uint16_t* d_fp16, int N, int K) {
    if (!c || !name || !q || !d_fp16) { set_error("invalid argument"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    const std::string n = strip(name);
    auto pt = c->parts.find(n);
    if (pt == c->parts.end()) { set_error("no Q8_0 decoder tensor named " + n); return ERR_NOT_FOUND; }
    const Part& p = pt->second;
    if (N != p.rows || K != p.m->K) {
        set_error(n + ": expected [" + std::to_string(p.rows) + ", " + std::to_string(p.m->K) + "]");
        return ERR_ARGUMENT;
    }
    RC(fill_rows_q8(c, p, q, d_fp16));
    c->have.insert(n);
    return OK;
}

int laya_decoder_missing(laya_decoder* c, char* names, int cap, int* missing) {
    if (!c || !missing) { set_error("null argument"); return ERR_ARGUMENT; }
    std::string out;
    int m = 0;
    for (auto& p : c->parts)
        if (!c->have.count(p.first)) { ++m; out += p.first + "\n"; }
    for (auto& v : c->vecs)
        if (!c->have.count(v.first)) { ++m; out += v.first + "\n"; }
    *missing = m;
    if (names && cap > 0) {
        const size_t k = std::min(out.size(), static_cast<size_t>(cap - 1));
        memcpy(names, out.data(), k);
        names[k] = 0;
    }
    return OK;
}

int laya_decoder_forward_device(laya_decoder* c, const int32_t* ids, const int32_t* seq_len, int n_seq,
                                const int32_t* label_ids, int n_labels, float* hidden, float* logits) {
    if (!c || !ids || !seq_len) { set_error("null argument"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    RC(ready(c));
    int T = 0;
    long long pairs = 0;
    RC(stage(c, nullptr, seq_len, n_seq, label_ids, n_labels, &T, &pairs));
    c->ids = const_cast<int32_t*>(ids);
    RC(forward_body(c, T, n_seq, pairs, n_labels, hidden, logits));
    if (c->profiling) RC(collect_profile(c));
    return OK;
}

int laya_decoder_forward(laya_decoder* c, const int32_t* ids, const int32_t* seq_len, int n_seq,
                         const int32_t* label_ids, int n_labels, float* hidden, float* logits) {
    if (!c || !ids || !seq_len) { set_error("null argument"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    RC(ready(c));
    int T = 0;
    long long pairs = 0;
    RC(stage(c, ids, seq_len, n_seq, label_ids, n_labels, &T, &pairs));
    const size_t nl = static_cast<size_t>(n_seq) * n_labels;
    RC(ensure_logits(c, nl));
    RC(forward_body(c, T, n_seq, pairs, n_labels, nullptr, logits && n_labels ? c->logit_buf : nullptr));
    if (hidden)
        LAYA_CUDA(cudaMemcpyAsync(hidden, c->hid, static_cast<size_t>(n_seq) * c->d.hidden * sizeof(float),
                                  cudaMemcpyDeviceToHost, c->stream));
    if (logits && n_labels)
        LAYA_CUDA(cudaMemcpyAsync(logits, c->logit_buf, nl * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    RC(check_device_error(c));
    if (c->profiling) RC(collect_profile(c));
    return OK;
}

int laya_decoder_state_create(laya_decoder* c, int capacity, laya_decoder_state** out) {
    if (!c || !out || capacity < 0) { set_error("invalid argument"); return ERR_ARGUMENT; }
    *out = nullptr;
    DeviceGuard g(c->device);
    return state_new(c, capacity, out);
}

int laya_decoder_state_destroy(laya_decoder_state* st) {
    if (!st) return OK;
    if (st->dec) {
        DeviceGuard g(st->dec->device);
        state_free(st);
    } else {
        delete st;
    }
    return OK;
}

int laya_decoder_state_length(const laya_decoder_state* st, int* length) {
    if (!st || !length) { set_error("null argument"); return ERR_ARGUMENT; }
    *length = st->length;
    return OK;
}

int laya_decoder_state_bytes(const laya_decoder_state* st, int64_t* bytes) {
    if (!st || !bytes) { set_error("null argument"); return ERR_ARGUMENT; }
    *bytes = st->dec ? static_cast<int64_t>(st->bytes) : 0;
    return OK;
}

int laya_decoder_state_clone(laya_decoder_state* st, laya_decoder_state** out) {
    if (!st || !out) { set_error("null argument"); return ERR_ARGUMENT; }
    *out = nullptr;
    if (!st->dec) { set_error("the state's decoder was destroyed"); return ERR_ARGUMENT; }
    laya_decoder* c = st->dec;
    DeviceGuard g(c->device);
    laya_decoder_state* copy = nullptr;
    RC(state_new(c, st->capacity, &copy));
    const int rc = state_copy(c, st, copy);
    if (rc != OK) { state_free(copy); return rc; }
    *out = copy;
    return OK;
}

int laya_decoder_state_save(laya_decoder_state* st, laya_decoder_mark** out) {
    if (!st || !out) { set_error("null argument"); return ERR_ARGUMENT; }
    *out = nullptr;
    if (!st->dec) { set_error("the state's decoder was destroyed"); return ERR_ARGUMENT; }
    laya_decoder* c = st->dec;
    DeviceGuard g(c->device);
    laya_decoder_mark* m = new laya_decoder_mark();
    m->dec = c;
    m->length = st->length;
    m->bytes = st->fixed;
    if (m->bytes) {
        void* p = nullptr;
        cudaError_t e = pool_alloc(c, &p, m->bytes);
        if (e == cudaSuccess) e = cudaMemcpyAsync(p, st->block, m->bytes, cudaMemcpyDeviceToDevice, c->stream);
        m->block = static_cast<char*>(p);
        if (e != cudaSuccess) {
            if (p) cudaFreeAsync(p, c->stream);
            delete m;
            return cuda_fail(e, "state save");
        }
    }
    c->marks.insert(m);
    *out = m;
    return OK;
}

int laya_decoder_state_rewind(laya_decoder_state* st, const laya_decoder_mark* m) {
    if (!st || !m) { set_error("null argument"); return ERR_ARGUMENT; }
    if (!st->dec || m->dec != st->dec) { set_error("the mark belongs to another decoder"); return ERR_ARGUMENT; }
    if (m->length > st->length) { set_error("a mark can only rewind, not advance"); return ERR_ARGUMENT; }
    laya_decoder* c = st->dec;
    DeviceGuard g(c->device);
    if (m->bytes) LAYA_CUDA(cudaMemcpyAsync(st->block, m->block, m->bytes, cudaMemcpyDeviceToDevice, c->stream));
    st->length = m->length;
    return OK;
}

int laya_decoder_mark_destroy(laya_decoder_mark* m) {
    if (!m) return OK;
    if (m->dec) {
        DeviceGuard g(m->dec->device);
        if (m->block) cudaFreeAsync(m->block, m->dec->stream);
        m->dec->marks.erase(m);
    }
    delete m;
    return OK;
}

int laya_decoder_forward_states(laya_decoder* c, const int32_t* ids, const int32_t* seq_len, int n_seq,
                                laya_decoder_state* const* states, const int32_t* readout, const int32_t* n_checkpoints,
                                const int32_t* checkpoints, laya_decoder_state** snapshots, const int32_t* label_ids,
                                int n_labels, float* hidden, float* logits) {
    (void)readout;   // every sequence's row is computed; rows of sequences without readout are not needed
    if (!c || !ids || !seq_len || !states) { set_error("null argument"); return ERR_ARGUMENT; }
    if (n_seq <= 0 || n_seq > c->d.max_seqs) { set_error("sequence count outside 1..max_seqs"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    RC(ready(c));
    // validate everything before any device work: a rejected call leaves every state as it was
    std::set<const laya_decoder_state*> seen;
    int n_snap = 0, longest = 0;
    long long T = 0;
    for (int s = 0; s < n_seq; ++s) {
        const laya_decoder_state* st = states[s];
        if (!st || st->dec != c) { set_error("a state is null or belongs to another decoder"); return ERR_ARGUMENT; }
        if (!seen.insert(st).second) { set_error("two sequences continue the same state"); return ERR_ARGUMENT; }
        if (seq_len[s] <= 0) { set_error("every sequence needs at least one token"); return ERR_ARGUMENT; }
        if (static_cast<long long>(st->length) + seq_len[s] > INT32_MAX / 2) { set_error("state too long"); return ERR_ARGUMENT; }
        const int n = n_checkpoints ? n_checkpoints[s] : 0;
        if (n < 0 || (n > 0 && (!checkpoints || !snapshots))) { set_error("invalid checkpoint list"); return ERR_ARGUMENT; }
        for (int k = 0; k < n; ++k) {
            const int cp = checkpoints[n_snap + k];
            const int prev = k ? checkpoints[n_snap + k - 1] : 0;
            if (cp <= prev || cp > seq_len[s]) { set_error("checkpoints must ascend strictly within 1..seq_len"); return ERR_ARGUMENT; }
        }
        n_snap += n;
        T += seq_len[s];
        longest = std::max(longest, st->length + seq_len[s]);
    }
    if (T > c->d.max_tokens) { set_error("more tokens than max_tokens"); return ERR_ARGUMENT; }
    for (long long t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= c->d.vocab) { set_error("token id outside the vocabulary"); return ERR_OUT_OF_RANGE; }
    for (int l = 0; l < n_labels; ++l)
        if (!label_ids || label_ids[l] < 0 || label_ids[l] >= c->d.vocab) { set_error("label id outside the vocabulary"); return ERR_OUT_OF_RANGE; }

    for (int s = 0; s < n_seq; ++s) RC(state_grow(c, states[s], states[s]->length + seq_len[s]));
    if (n_full_layers(c) > 0) RC(ensure_rope(c, longest));
    std::vector<laya_decoder_state*> snaps;
    auto fail = [&](int rc) {
        for (laya_decoder_state* x : snaps) state_free(x);
        return rc;
    };
    for (int s = 0, k0 = 0; s < n_seq; ++s) {
        const int n = n_checkpoints ? n_checkpoints[s] : 0;
        for (int k = 0; k < n; ++k) {
            laya_decoder_state* x = nullptr;
            const int rc = state_new(c, states[s]->length + checkpoints[k0 + k], &x);
            if (rc != OK) return fail(rc);
            snaps.push_back(x);
        }
        k0 += n;
    }
    StateView sv;
    sv.states = states;
    sv.n_cp = n_checkpoints;
    sv.cps = checkpoints;
    sv.snaps = snaps.data();
    sv.n_snap = n_snap;
    int Ti = 0;
    long long pairs = 0;
    int rc = stage(c, ids, seq_len, n_seq, label_ids, n_labels, &Ti, &pairs, &sv);
    const size_t nl = static_cast<size_t>(n_seq) * n_labels;
    if (rc == OK) rc = ensure_logits(c, nl);
    if (rc == OK) rc = forward_body(c, Ti, n_seq, pairs, n_labels, nullptr, logits && n_labels ? c->logit_buf : nullptr);
    c->with_states = false;
    c->cur_snaps = 0;
    // snapshots take their sequence's keys and values up to the checkpoint (SnapshotKeysAndValues, :734-749)
    const size_t row = sizeof(__half) * static_cast<size_t>(c->d.kv_heads) * c->d.head_dim;
    for (int s = 0, k0 = 0; s < n_seq && rc == OK; ++s) {
        const int n = n_checkpoints ? n_checkpoints[s] : 0;
        for (int k = 0; k < n && rc == OK; ++k) {
            laya_decoder_state* x = snaps[k0 + k];
            const size_t len = static_cast<size_t>(states[s]->length) + checkpoints[k0 + k];
            for (int i = 0; i < c->d.layers && rc == OK; ++i) {
                if (c->kinds[i] != LAYA_DECODER_FULL) continue;
                cudaError_t e = cudaMemcpyAsync(x->k[i], states[s]->k[i], row * len, cudaMemcpyDeviceToDevice, c->stream);
                if (e == cudaSuccess) e = cudaMemcpyAsync(x->v[i], states[s]->v[i], row * len, cudaMemcpyDeviceToDevice, c->stream);
                if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpyAsync");
            }
            x->length = static_cast<int>(len);
        }
        k0 += n;
    }
    if (rc == OK && hidden) {
        cudaError_t e = cudaMemcpyAsync(hidden, c->hid, static_cast<size_t>(n_seq) * c->d.hidden * sizeof(float),
                                        cudaMemcpyDeviceToHost, c->stream);
        if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpyAsync");
    }
    if (rc == OK && logits && n_labels) {
        cudaError_t e = cudaMemcpyAsync(logits, c->logit_buf, nl * sizeof(float), cudaMemcpyDeviceToHost, c->stream);
        if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpyAsync");
    }
    if (rc == OK) rc = check_device_error(c);
    if (rc != OK) return fail(rc);
    for (int s = 0; s < n_seq; ++s) states[s]->length += seq_len[s];
    for (int k = 0; k < n_snap; ++k) snapshots[k] = snaps[k];
    if (c->profiling) RC(collect_profile(c));
    return OK;
}

int laya_decoder_logits(laya_decoder* c, const float* hidden, int rows, const int32_t* ids, int n_ids, float* logits) {
    if (!c || !hidden || !ids || !logits || rows <= 0 || n_ids <= 0) { set_error("invalid argument"); return ERR_ARGUMENT; }
    if (rows > c->d.max_seqs) { set_error("more rows than max_seqs"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    if (!c->have.count("embed_tokens.weight")) { set_error("missing tensor embed_tokens.weight"); return ERR_NOT_FOUND; }
    for (int i = 0; i < n_ids; ++i)
        if (ids[i] < 0 || ids[i] >= c->d.vocab) { set_error("label id outside the vocabulary"); return ERR_OUT_OF_RANGE; }
    const int h = c->d.hidden;
    const size_t nl = static_cast<size_t>(rows) * n_ids;
    RC(ensure_logits(c, nl));
    int32_t* lab = nullptr;
    LAYA_CUDA(cudaMalloc(&lab, sizeof(int32_t) * n_ids));
    cudaError_t e = cudaMemcpyAsync(lab, ids, sizeof(int32_t) * n_ids, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(c->hid, hidden, sizeof(float) * rows * h, cudaMemcpyHostToDevice, c->stream);
    int rc = e == cudaSuccess ? q8::quantize_activations(c->hid, rows, h, h, c->qlast, c->dlast, c->ldl, c->stream)
                              : cuda_fail(e, "cudaMemcpyAsync");
    if (rc == OK) {
        dec::LogitArgs lg{};
        lg.n_seq = rows; lg.n_labels = n_ids; lg.n = h; lg.vocab = c->d.vocab;
        lg.qx = c->qlast; lg.dx = c->dlast; lg.ldx = c->ldl;
        lg.qw = c->table.q; lg.dw = c->table.d; lg.ldw = c->table.ldw;
        lg.labels = lab; lg.logits = c->logit_buf; lg.err = c->err;
        rc = dec_q8_logits(lg, c->stream);
    }
    if (rc == OK) {
        e = cudaMemcpyAsync(logits, c->logit_buf, nl * sizeof(float), cudaMemcpyDeviceToHost, c->stream);
        if (e != cudaSuccess) rc = cuda_fail(e, "cudaMemcpyAsync");
    }
    cudaStreamSynchronize(c->stream);
    cudaFree(lab);
    if (rc != OK) return rc;
    return check_device_error(c);
}

int laya_decoder_layer(laya_decoder* c, int layer, float* hidden, const int32_t* seq_len, int n_seq, float* mixer) {
    if (!c || !hidden || !seq_len) { set_error("null argument"); return ERR_ARGUMENT; }
    if (layer < 0 || layer >= c->d.layers) { set_error("layer index out of range"); return ERR_OUT_OF_RANGE; }
    DeviceGuard g(c->device);
    RC(ready(c));
    int T = 0;
    long long pairs = 0;
    RC(stage_input_rows(c, seq_len, n_seq, &T, &pairs));
    const size_t n = static_cast<size_t>(T) * c->d.hidden;
    LAYA_CUDA(cudaMemcpyAsync(c->x, hidden, n * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    RC(run_layer(c, layer, T, n_seq, pairs, mixer != nullptr));
    LAYA_CUDA(cudaMemcpyAsync(hidden, c->x, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    if (mixer) LAYA_CUDA(cudaMemcpyAsync(mixer, c->mix, n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    return check_device_error(c);
}

int laya_decoder_set_chunked_delta_rule(laya_decoder* c, int enabled) {
    if (!c) { set_error("null decoder"); return ERR_ARGUMENT; }
    c->chunked_rule = enabled != 0;
    return OK;
}

int laya_decoder_record_enable(laya_decoder* c, int enabled) {
    if (!c) { set_error("null decoder"); return ERR_ARGUMENT; }
    c->record = enabled != 0;
    return OK;
}

int laya_decoder_record_get(laya_decoder* c, const char* name, float* host, int64_t count) {
    if (!c || !name || !host) { set_error("invalid argument"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    auto it = c->rec.find(name);
    if (it == c->rec.end()) { set_error(std::string("nothing recorded as ") + name); return ERR_NOT_FOUND; }
    if (count < static_cast<int64_t>(it->second.count)) { set_error("host buffer too small"); return ERR_ARGUMENT; }
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    LAYA_CUDA(cudaMemcpy(host, it->second.p, it->second.count * sizeof(float), cudaMemcpyDeviceToHost));
    return OK;
}

int laya_decoder_launches(laya_decoder* c, long long* count) {
    if (!c || !count) { set_error("null argument"); return ERR_ARGUMENT; }
    *count = launches();
    return OK;
}

int laya_decoder_set_profiling(laya_decoder* c, int enabled) {
    if (!c) { set_error("null decoder"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    RC(collect_profile(c));
    c->profiling = enabled != 0;
    for (int k = 0; k < 3; ++k) { c->prof_ms[k] = c->prof_ops[k] = 0; c->prof_n[k] = 0; }
    return OK;
}

int laya_decoder_profile(laya_decoder* c, int kind, double* ms, double* ops, long long* n) {
    if (!c) { set_error("null decoder"); return ERR_ARGUMENT; }
    if (kind < 0 || kind > 2) { set_error("profile kind is 0 (products), 1 (delta rule) or 2 (attention)"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    RC(collect_profile(c));
    if (ms) *ms = c->prof_ms[kind];
    if (ops) *ops = c->prof_ops[kind];
    if (n) *n = c->prof_n[kind];
    c->prof_ms[kind] = c->prof_ops[kind] = 0;
    c->prof_n[kind] = 0;
    return OK;
}

}  // extern "C"
