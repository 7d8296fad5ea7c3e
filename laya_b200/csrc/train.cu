// train.cu — the fine-tuning step behind include/laya_train.h.
//
// Host C++ only: it owns the trainer's device memory and orders the kernels of gemm_bf16.cu, flash.cu and
// train_kernels.cu into TrainableDecisionModel's forward and backward (Laya.Training/TrainableDecisionModel.cs:
// 248-640), RlcdObjective.Compute (RlcdObjective.cs:57-155), Gradients.ClipByGlobalNorm + AdamW.Step (AdamW.cs:
// 29-130), plus a bucketed NCCL gradient allreduce for data parallelism.
//
// Device state:
//   parameters   one flat fp32 master buffer in a fixed order — embeddings, encoder layers 0..L-1, final norm (group
//                0), then type embedding, head layers, scorer, action head (group 1) — each tensor 256-byte aligned;
//                a bf16 copy of it for the products; fp32 gradients; AdamW m and v.  Trainable encoder parameters are
//                a suffix of group 0, so each group's update is one contiguous range.
//   tape         every activation the backward reads stays in HBM from the forward (the reference recomputes each
//                layer instead, TrainableDecisionModel.cs:551-557): layer inputs and residual midpoints in fp32,
//                the product operands (normalised rows, qkv, attention context, GeGLU input and output) in bf16,
//                LayerNorm mean/rstd and the attention row log-sum-exp in fp32.
//   batches      laya_batch objects: ids, segment table, attention tile list, marker rows, targets and noise draws.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/laya_train.h"
#include "common.cuh"
#include "internal.h"
#include "safetensors.h"
#include "train.h"

using bf16 = __nv_bfloat16;

namespace laya {
namespace {

constexpr size_t NONE = static_cast<size_t>(-1);
constexpr size_t BUCKET_ELEMS = 25u * 1000u * 1000u / 4u;   // 25 MB of fp32 gradients per allreduce
constexpr int MAX_GROUPS = 16;                               // noise groups a batch can carry
constexpr size_t DMASK_MAX = size_t(1) << 30;                  // the head layers' dropout decisions, at most
constexpr size_t DS_SCRATCH_MAX = size_t(2) << 30;            // the attention backward's dS scratch, at most

#define RC(x)                      \
    do {                           \
        int rc_ = (x);             \
        if (rc_ != OK) return rc_; \
    } while (0)

// Ops.Mix and TrainableDecisionModel.Salt (Ops.cs:236-241; TrainableDecisionModel.cs:422).
uint64_t mix64(uint64_t seed, uint64_t salt) {
    uint64_t z = seed ^ (salt * 0xD1B54A32D192ED03ull + 0x8CB92BA72F3D8DD7ull);
    z = (z ^ (z >> 33)) * 0xFF51AFD7ED558CCDull;
    return z ^ (z >> 33);
}
uint64_t salt(uint64_t seed, int layer, int site) { return mix64(seed, static_cast<uint64_t>(layer) * 16 + site + 1); }

struct Param {
    std::string name;
    int64_t rows, cols;
    size_t off;
    int group;
    bool trainable;
    std::vector<int64_t> shape;   // as uploaded (else [cols] for a single row, [rows, cols] otherwise)
    int stored = LAYA_F32;        // the dtype it was uploaded in: what a checkpoint writes it back as
};
struct EncP { size_t n1, qkv, wo, n2, wi, wo2; };
struct HeadP { size_t n1w, n1b, inw, inb, outw, outb, n2w, n2b, l1w, l1b, l2w, l2b; };

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

// NCCL through dlopen: the library has no link-time dependency on it, and a process that already loaded NCCL (a
// framework, or the C# host's own) shares that copy.
struct Nccl {
    void* lib = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    const char* (*getErrorString)(ncclResult_t) = nullptr;
};
Nccl g_nccl;
std::mutex g_nccl_mu;

int load_nccl() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.lib) return OK;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) { set_error("NCCL (libnccl.so.2) could not be loaded"); return ERR_COMM; }
    Nccl n;
    n.lib = h;
    n.getUniqueId = reinterpret_cast<decltype(n.getUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    n.commInitRank = reinterpret_cast<decltype(n.commInitRank)>(dlsym(h, "ncclCommInitRank"));
    n.allReduce = reinterpret_cast<decltype(n.allReduce)>(dlsym(h, "ncclAllReduce"));
    n.commDestroy = reinterpret_cast<decltype(n.commDestroy)>(dlsym(h, "ncclCommDestroy"));
    n.getErrorString = reinterpret_cast<decltype(n.getErrorString)>(dlsym(h, "ncclGetErrorString"));
    if (!n.getUniqueId || !n.commInitRank || !n.allReduce || !n.commDestroy || !n.getErrorString) {
        set_error("NCCL library lacks an expected entry point");
        return ERR_COMM;
    }
    g_nccl = n;
    return OK;
}
int nccl_fail(ncclResult_t r, const char* what) {
    set_error(std::string(what) + ": " + (g_nccl.getErrorString ? g_nccl.getErrorString(r) : "NCCL error"));
    return ERR_COMM;
}

}  // namespace
}  // namespace laya

using laya::EncP;
using laya::HeadP;
using laya::NONE;
using laya::OK;
using laya::Param;

struct laya_batch {
    laya_trainer* owner = nullptr;   // identity only: a batch may outlive its trainer and still be destroyed
    int device = 0;
    uint64_t id = 0;                 // unique over the process: a new batch at a freed one's address is not it
    uint64_t version = 0;            // bumped by every laya_batch_set
    double pairs_global = 0, pairs_local = 0;   // visible (query, key) pairs: full segments; the sliding window
    int T = 0, n = 0, M = 0, tiles = 0, groups = 0;
    // device fields (one allocation, layout fixed by capacity)
    void* dev = nullptr;
    void* host = nullptr;   // pinned staging of the same layout
    size_t bytes = 0;
    cudaEvent_t staged = nullptr;
    int32_t *ids, *seg_start, *seg_len, *qtype, *tok_item, *tile_item, *tile_p0, *n_tiles, *marker_rows, *mk_start,
        *mk_count, *tq_item, *tq_p0, *n_tq, *tp_item, *tp_p0, *n_tp;
    int tq = 0;                      // 128-row query tiles (tcgen05 attention)
    int tp = 0;                      // 256-row pair tiles (the two-tile attention forward), longest segments first
    float* targets;
    double* draws;
    size_t o_ids, o_seg_start, o_seg_len, o_qtype, o_tok_item, o_tile_item, o_tile_p0, o_n_tiles, o_marker_rows,
        o_mk_start, o_mk_count, o_tq_item, o_tq_p0, o_n_tq, o_tp_item, o_tp_p0, o_n_tp, o_targets, o_draws;
};

struct Comm {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    cudaStream_t stream = nullptr;
    cudaEvent_t ready = nullptr, done = nullptr;
    std::vector<std::pair<size_t, size_t>> buckets;   // [begin, end) from the top of the buffer down
    size_t next = 0;                                  // first bucket not yet issued this window
    bool active = false;                              // buckets are being issued during this backward
    bool reduced = false;                             // this window's gradients have been summed
};

struct laya_trainer {
    int device = 0;
    laya_model_desc d{};
    laya_train_desc td{};
    int H = 0, I = 0, L = 0, heads = 0, hd = 0, HL = 0, HH = 0, FF = 0, V = 0, window = 0, maxpos = 0;
    float eps = 1e-5f;
    std::vector<char> global;
    // parameters
    std::vector<Param> params;
    std::unordered_map<std::string, int> index;
    size_t P = 0, enc_train_begin = 0, enc_end = 0, head_begin = 0;
    size_t tok_emb = 0, emb_norm = 0, final_norm = 0, type_emb = 0, sc0w = 0, sc0b = 0, sc1w = 0, sc1b = 0, sc3w = 0,
           sc3b = 0;
    std::vector<EncP> enc;
    std::vector<HeadP> head;
    std::vector<size_t> head_start;   // first element of each head layer's parameters
    size_t scorer_start = 0;
    int first_trainable = 0;
    bool emb_trainable = true;
    float *master = nullptr, *grad = nullptr, *m = nullptr, *v = nullptr;
    bf16* shadow = nullptr;
    bf16* shadow_lo = nullptr;   // accurate forward: master − bf16(master)
    bool precise = true;
    // capacity
    int Tc = 0, Mc = 0, Nc = 0, tiles_cap = 0;
    // tape
    std::vector<float*> X, X1, mean1, rstd1, mean2, rstd2, lse;
    std::vector<bf16*> n1, qkv, ctx, n2, wide, act;          // bf16; qkv with q, k rotated (wide: BF16 forward only)
    std::vector<bf16*> n1lo, ctxlo, n2lo, actlo;             // accurate forward: low parts
    std::vector<float*> wide32;                              // accurate forward: fp32 GeGLU input
    float* ws_qkv32 = nullptr;                               // accurate forward: fp32 qkv of the current layer
    bf16* ws_qkvlo = nullptr;                                //   and the low parts of its rotated q, k, v
    float *emb_mean = nullptr, *emb_rstd = nullptr, *f_mean = nullptr, *f_rstd = nullptr;
    std::vector<float*> HIN, HX1, hm1, hr1, hm2, hr2, hlse;
    std::vector<bf16*> hn1, hqkv, hctx, hn2, hpre, hact;
    std::vector<bf16*> hn1lo, hctxlo, hn2lo, hactlo;
    std::vector<float*> hpre32;
    bf16* sn16 = nullptr;
    bf16* snlo = nullptr;
    float *smean = nullptr, *srstd = nullptr, *spre = nullptr, *logits = nullptr, *dlog = nullptr;
    // workspace
    float *R32 = nullptr, *dH = nullptr, *dN = nullptr, *dbig32 = nullptr, *dsum = nullptr, *dsn = nullptr;
    uint8_t* ds = nullptr;   // the attention backward's dS scratch (null when it would exceed DS_SCRATCH_MAX)
    int ds_nq = 0;
    // the head layers' attention dropout decisions, one bit per probability, drawn by each training forward for itself
    // and its backward (null when they would exceed DMASK_MAX: the kernels then evaluate the hash per probability)
    uint32_t* dmask = nullptr;
    int dmask_w = 0, dmask_rows = 0;
    size_t dmask_layer = 0;   // words per head layer
    // the decisions are drawn on a second stream while the encoder layers run (whose kernels leave most issue slots
    // idle); mask_begin orders them after the previous step's backward, mask_done before the head layers
    cudaStream_t mask_stream = nullptr;
    cudaEvent_t mask_begin = nullptr, mask_done = nullptr;
    bool masks_pending = false;
    float* ln_part = nullptr;                                // LayerNorm backward: per-CTA dγ/dβ partials
    bf16 *d16 = nullptr, *dctx16 = nullptr, *dqkv16 = nullptr, *dbig16 = nullptr, *dpre16 = nullptr;
    float *cos_g = nullptr, *sin_g = nullptr, *cos_l = nullptr, *sin_l = nullptr;
    double* red = nullptr;   // [0] Σg², [1] gradient factor, [2] norm, [4..7] objective results, [8..] Σg² partials
    double* rl_scratch = nullptr;
    double* h_red = nullptr;   // pinned
    int* err = nullptr;
    cudaStream_t stream = nullptr, own = nullptr;
    double lr[2] = {0, 0};
    int64_t steps = 0;
    int micro = 0;
    // last forward: the batch it ran on (id and contents version) and its mode
    uint64_t fwd_id = 0, fwd_version = 0;
    bool fwd_training = false;
    uint64_t fwd_seed = 0;
    bool have_logits = false, have_dlogits = false;
    Comm comm;
    // profiling: CUDA events around each product (kind 0) and attention forward (1) / backward (2) launch
    bool profiling = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev_pool;
    std::vector<std::pair<int, double>> ev_work;   // (kind, algorithmic FLOPs) of each used event pair
    double prof_ms[3] = {0, 0, 0}, prof_flops[3] = {0, 0, 0};
    long long prof_n[3] = {0, 0, 0};
    std::vector<void*> allocs;
};

namespace laya {
namespace {

int dalloc(laya_trainer* t, void** p, size_t bytes) {
    bytes = (bytes + 255) & ~size_t(255);
    if (bytes == 0) bytes = 256;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    t->allocs.push_back(*p);
    return OK;
}
template <class T>
int dalloc_t(laya_trainer* t, T** p, size_t count) {
    return dalloc(t, reinterpret_cast<void**>(p), count * sizeof(T));
}

int check_device_error(laya_trainer* t) {
    int h = 0;
    LAYA_CUDA(cudaMemcpyAsync(&h, t->err, sizeof(int), cudaMemcpyDeviceToHost, t->stream));
    LAYA_CUDA(cudaStreamSynchronize(t->stream));
    if (h != 0) {
        LAYA_CUDA(cudaMemsetAsync(t->err, 0, sizeof(int), t->stream));
        LAYA_CUDA(cudaStreamSynchronize(t->stream));
        if (h == LAYA_DEV_ERR_TIMEOUT) { set_error("a device-side wait timed out"); return ERR_DEVICE_TIMEOUT; }
        set_error("index out of range on the device");
        return ERR_OUT_OF_RANGE;
    }
    return OK;
}

// Runs `launch` between two CUDA events when profiling is on, charging `flops` algorithmic FLOPs to `kind`.
template <class F>
int timed(laya_trainer* t, int kind, double flops, F&& launch) {
    if (!t->profiling) return launch();
    if (t->ev_work.size() == t->ev_pool.size()) {
        cudaEvent_t e0, e1;
        LAYA_CUDA(cudaEventCreate(&e0));
        LAYA_CUDA(cudaEventCreate(&e1));
        t->ev_pool.push_back({e0, e1});
    }
    auto& ev = t->ev_pool[t->ev_work.size()];
    LAYA_CUDA(cudaEventRecord(ev.first, t->stream));
    const int rc = launch();
    LAYA_CUDA(cudaEventRecord(ev.second, t->stream));
    t->ev_work.push_back({kind, flops});
    return rc;
}

int collect_profile(laya_trainer* t) {
    if (t->ev_work.empty()) return OK;
    LAYA_CUDA(cudaStreamSynchronize(t->stream));
    for (size_t i = 0; i < t->ev_work.size(); ++i) {
        float ms = 0;
        LAYA_CUDA(cudaEventElapsedTime(&ms, t->ev_pool[i].first, t->ev_pool[i].second));
        const int k = t->ev_work[i].first;
        t->prof_ms[k] += ms;
        t->prof_flops[k] += t->ev_work[i].second;
        t->prof_n[k] += 1;
    }
    t->ev_work.clear();
    return OK;
}

// ------------------------------------------------------------------------------------------------ registry
// The parameters TrainableDecisionModel reads (TrainableDecisionModel.cs:111-178), in buffer order.
void add_param(laya_trainer* t, const std::string& name, int64_t rows, int64_t cols, int group) {
    Param p{name, rows, cols, t->P, group, true};
    p.shape = rows == 1 ? std::vector<int64_t>{cols} : std::vector<int64_t>{rows, cols};
    t->index[name] = static_cast<int>(t->params.size());
    t->params.push_back(p);
    const size_t n = static_cast<size_t>(rows) * cols;
    t->P += (n + 63) / 64 * 64;   // 256-byte aligned fp32, 128-byte aligned bf16
}
size_t off(laya_trainer* t, const std::string& name) { return t->params[t->index.at(name)].off; }

void build_registry(laya_trainer* t) {
    const int H = t->H;
    const std::string e = "encoder.", lp = "encoder.layers.";
    add_param(t, e + "embeddings.tok_embeddings.weight", t->V, H, 0);
    add_param(t, e + "embeddings.norm.weight", 1, H, 0);
    for (int l = 0; l < t->L; ++l) {
        const std::string p = lp + std::to_string(l) + ".";
        if (l > 0) add_param(t, p + "attn_norm.weight", 1, H, 0);
        add_param(t, p + "attn.Wqkv.weight", 3 * H, H, 0);
        add_param(t, p + "attn.Wo.weight", H, H, 0);
        add_param(t, p + "mlp_norm.weight", 1, H, 0);
        add_param(t, p + "mlp.Wi.weight", 2 * t->I, H, 0);
        add_param(t, p + "mlp.Wo.weight", H, t->I, 0);
    }
    add_param(t, e + "final_norm.weight", 1, H, 0);
    t->enc_end = t->P;
    t->head_begin = t->P;
    add_param(t, "type_emb.weight", 3, H, 1);
    for (int l = 0; l < t->HL; ++l) {
        const std::string p = "head.layers." + std::to_string(l) + ".";
        add_param(t, p + "norm1.weight", 1, H, 1);
        add_param(t, p + "norm1.bias", 1, H, 1);
        add_param(t, p + "self_attn.in_proj_weight", 3 * H, H, 1);
        add_param(t, p + "self_attn.in_proj_bias", 1, 3 * H, 1);
        add_param(t, p + "self_attn.out_proj.weight", H, H, 1);
        add_param(t, p + "self_attn.out_proj.bias", 1, H, 1);
        add_param(t, p + "norm2.weight", 1, H, 1);
        add_param(t, p + "norm2.bias", 1, H, 1);
        add_param(t, p + "linear1.weight", t->FF, H, 1);
        add_param(t, p + "linear1.bias", 1, t->FF, 1);
        add_param(t, p + "linear2.weight", H, t->FF, 1);
        add_param(t, p + "linear2.bias", 1, H, 1);
    }
    add_param(t, "scorer.0.weight", 1, H, 1);
    add_param(t, "scorer.0.bias", 1, H, 1);
    add_param(t, "scorer.1.weight", H, H, 1);
    add_param(t, "scorer.1.bias", 1, H, 1);
    add_param(t, "scorer.3.weight", 1, H, 1);
    add_param(t, "scorer.3.bias", 1, 1, 1);
    add_param(t, "act_head.0.weight", t->d.act_hidden, H + 4, 1);
    add_param(t, "act_head.0.bias", 1, t->d.act_hidden, 1);
    add_param(t, "act_head.2.weight", t->d.n_act, t->d.act_hidden, 1);
    add_param(t, "act_head.2.bias", 1, t->d.n_act, 1);

    t->tok_emb = off(t, e + "embeddings.tok_embeddings.weight");
    t->emb_norm = off(t, e + "embeddings.norm.weight");
    t->final_norm = off(t, e + "final_norm.weight");
    t->type_emb = off(t, "type_emb.weight");
    t->enc.resize(t->L);
    for (int l = 0; l < t->L; ++l) {
        const std::string p = lp + std::to_string(l) + ".";
        EncP& q = t->enc[l];
        q.n1 = l > 0 ? off(t, p + "attn_norm.weight") : NONE;
        q.qkv = off(t, p + "attn.Wqkv.weight");
        q.wo = off(t, p + "attn.Wo.weight");
        q.n2 = off(t, p + "mlp_norm.weight");
        q.wi = off(t, p + "mlp.Wi.weight");
        q.wo2 = off(t, p + "mlp.Wo.weight");
    }
    t->head.resize(t->HL);
    t->head_start.resize(t->HL);
    for (int l = 0; l < t->HL; ++l) {
        const std::string p = "head.layers." + std::to_string(l) + ".";
        HeadP& q = t->head[l];
        q.n1w = off(t, p + "norm1.weight"); q.n1b = off(t, p + "norm1.bias");
        q.inw = off(t, p + "self_attn.in_proj_weight"); q.inb = off(t, p + "self_attn.in_proj_bias");
        q.outw = off(t, p + "self_attn.out_proj.weight"); q.outb = off(t, p + "self_attn.out_proj.bias");
        q.n2w = off(t, p + "norm2.weight"); q.n2b = off(t, p + "norm2.bias");
        q.l1w = off(t, p + "linear1.weight"); q.l1b = off(t, p + "linear1.bias");
        q.l2w = off(t, p + "linear2.weight"); q.l2b = off(t, p + "linear2.bias");
        t->head_start[l] = q.n1w;
    }
    t->sc0w = off(t, "scorer.0.weight"); t->sc0b = off(t, "scorer.0.bias");
    t->sc1w = off(t, "scorer.1.weight"); t->sc1b = off(t, "scorer.1.bias");
    t->sc3w = off(t, "scorer.3.weight"); t->sc3b = off(t, "scorer.3.bias");
    t->scorer_start = t->sc0w;

    // SetTrainableEncoderLayers (TrainableDecisionModel.cs:206-231)
    const int n = t->td.trainable_encoder_layers;
    const int trainable = n < 0 ? t->L : std::min(n, t->L);
    t->first_trainable = t->L - trainable;
    t->emb_trainable = n < 0 || n > t->L;   // null, or at least every layer: the embeddings train too
    t->enc_train_begin = t->enc_end;
    for (auto& p : t->params) {
        if (p.group != 0) continue;
        bool train;
        if (p.name.rfind("encoder.embeddings.", 0) == 0) train = t->emb_trainable;
        else if (p.name.rfind("encoder.final_norm.", 0) == 0) train = trainable > 0;
        else train = std::stoi(p.name.substr(15, p.name.find('.', 15) - 15)) >= t->first_trainable;
        p.trainable = train;
        if (train) t->enc_train_begin = std::min(t->enc_train_begin, p.off);
    }
}

// ------------------------------------------------------------------------------------------------ products
// out = A · Bᵀ in the three training layouts (gemm_bf16.cu): forward y = x·Wᵀ, input gradient dx = dy·W, weight
// gradient dW += dyᵀ·x.  W is [N, K] row-major everywhere.
// x_lo: the activation's low part in the accurate forward (the weight's comes from shadow_lo), else null.
int lin_fwd(laya_trainer* t, int T, int N, int K, const bf16* x, const bf16* x_lo, size_t w, const float* bias, int epi,
            void* out) {
    bf::Args a{T, N, K, x, K, 0, t->shadow + w, K, 0, bias, epi, out, N, t->err};
    if (x_lo) { a.A2 = x_lo; a.B2 = t->shadow_lo + w; }
    return timed(t, 0, 2.0 * T * N * K, [&] { return bf::gemm(a, t->stream); });
}
// The attention input in one product (EPI_QKV): q | k | v = x·Wᵀ (+ bias), q and k rotated at each row's segment
// position (cosv null: none), bf16 hi into `hi` and, with x_lo, the low parts into `lo`.  ERR_NOT_SUPPORTED when the
// product does not run on CTA pairs (then the caller writes fp32 and runs the prep pass).
int lin_qkv(laya_trainer* t, const laya_batch* b, int T, int N, int K, const bf16* x, const bf16* x_lo, size_t w,
            const float* bias, const float* cosv, const float* sinv, int rot_cols, bf16* hi, bf16* lo) {
    if (T <= 128 || (cosv && t->hd != 64)) return ERR_NOT_SUPPORTED;   // one-CTA sizes; rotation pairs (i, i + 32)
    bf::Args a{T, N, K, x, K, 0, t->shadow + w, K, 0, bias, bf::EPI_QKV, hi, N, t->err};
    if (x_lo) { a.A2 = x_lo; a.B2 = t->shadow_lo + w; a.out2 = lo; }
    a.tok_item = b->tok_item; a.seg_start = b->seg_start; a.cosv = cosv; a.sinv = sinv; a.rot_cols = rot_cols;
    int rc = ERR_NOT_SUPPORTED;
    const int t_rc = timed(t, 0, 2.0 * T * N * K, [&] {
        rc = bf::gemm(a, t->stream);
        return rc == ERR_NOT_SUPPORTED ? OK : rc;
    });
    return t_rc != OK ? t_rc : rc;
}
int lin_dx(laya_trainer* t, int T, int N, int K, const bf16* dy, size_t w, int epi, void* dx) {
    bf::Args a{T, K, N, dy, N, 0, t->shadow + w, K, 1, nullptr, epi, dx, K, t->err};
    return timed(t, 0, 2.0 * T * N * K, [&] { return bf::gemm(a, t->stream); });
}
int lin_dw(laya_trainer* t, int T, int N, int K, const bf16* dy, const bf16* x, size_t w) {
    bf::Args a{N, K, T, dy, N, 1, x, K, 1, nullptr, bf::EPI_F32_ADD, t->grad + w, K, t->err};
    a.ksplit_ok = 1;   // few output tiles over K = tokens: split K across the SMs
    return timed(t, 0, 2.0 * T * N * K, [&] { return bf::gemm(a, t->stream); });
}

fa::Args attn_args(laya_trainer* t, const laya_batch* b, const bf16* qkv, const bf16* qkv_lo, int heads, int window,
                   const float* cosv, const float* sinv, float dropout, uint64_t seed, bf16* out, bf16* out_lo,
                   float* lse) {
    fa::Args a{};
    a.qkv = qkv; a.qkv_lo = qkv_lo; a.out_lo = out_lo; a.ld = 3 * t->H; a.hidden = t->H; a.heads = heads;
    a.seg_start = b->seg_start; a.seg_len = b->seg_len;
    a.tile_item = b->tile_item; a.tile_p0 = b->tile_p0; a.n_tiles = b->n_tiles;
    a.window = window;
    a.scale = 1.0f / sqrtf(static_cast<float>(t->H / heads));
    a.cosv = cosv; a.sinv = sinv;
    a.dropout = dropout; a.keep = dropout > 0.f ? 1.0f / (1.0f - dropout) : 1.0f; a.seed = seed;
    a.out = out; a.ldo = t->H; a.lse = lse;
    a.dqkv = t->dqkv16; a.lddq = 3 * t->H; a.dsum = t->dsum; a.dout = t->dctx16;
    a.tq_item = b->tq_item; a.tq_p0 = b->tq_p0; a.n_tq = b->n_tq; a.max_tq = b->tq; a.T = b->T;
    a.tp_item = b->tp_item; a.tp_p0 = b->tp_p0; a.n_tp = b->n_tp; a.max_tp = b->tp;
    a.err = t->err;
    a.ds = t->ds; a.ds_nq = t->ds_nq;
    return a;
}

tr::Mask head_mask(laya_trainer* t, int l, int site) {
    const float p = t->fwd_training ? t->td.head_dropout : 0.0f;
    return tr::Mask{p, p > 0.f ? 1.0f / (1.0f - p) : 1.0f, salt(t->fwd_seed, l, site)};
}

tr::LnFwd ln_args(laya_trainer* t, int rows, const float* x, size_t w, size_t b, float eps, bf16* y16, bf16* y16lo,
                  float* y32, float* mean, float* rstd) {
    tr::LnFwd a{};
    a.rows = rows; a.n = t->H; a.x = x;
    a.w = t->master + w; a.b = b == NONE ? nullptr : t->master + b; a.eps = eps;
    a.y16 = y16; a.y16lo = y16lo; a.y32 = y32; a.mean = mean; a.rstd = rstd; a.err = t->err;
    return a;
}
template <class T>
T* at(const std::vector<T*>& v, int l) { return v.empty() ? nullptr : v[l]; }
tr::LnBwd lnb_args(laya_trainer* t, int rows, const float* x, const float* mean, const float* rstd, size_t w, size_t b,
                   const float* dy, float* dx, int accumulate) {
    tr::LnBwd a{};
    a.rows = rows; a.n = t->H; a.x = x; a.mean = mean; a.rstd = rstd; a.w = t->master + w;
    a.dy = dy; a.dx = dx; a.accumulate = accumulate;
    a.dw = t->grad + w; a.db = b == NONE ? nullptr : t->grad + b;
    a.part = t->ln_part;
    return a;
}

// ------------------------------------------------------------------------------------------------ forward
// EncoderLayerForward (TrainableDecisionModel.cs:361-414): LN → Wqkv → attention (RoPE, window) → Wo → +res → LN →
// Wi → GeGLU → Wo → +res.
int enc_forward(laya_trainer* t, const laya_batch* b, int l) {
    const int T = b->T, H = t->H, I = t->I;
    const EncP& p = t->enc[l];
    cudaStream_t s = t->stream;
    const bool pr = t->precise;
    bf16 *n1lo = at(t->n1lo, l), *n2lo = at(t->n2lo, l), *ctxlo = at(t->ctxlo, l), *actlo = at(t->actlo, l);
    if (p.n1 == NONE) {   // layer 0 has no attention norm (TrainableDecisionModel.cs:368-371)
        tr::LnFwd a = ln_args(t, T, t->X[l], t->emb_norm, NONE, t->eps, t->n1[l], n1lo, nullptr, nullptr, nullptr);
        a.identity = 1;
        RC(ln_fwd(a, s));
    } else {
        RC(ln_fwd(ln_args(t, T, t->X[l], p.n1, NONE, t->eps, t->n1[l], n1lo, nullptr, t->mean1[l], t->rstd1[l]), s));
    }
    const bool g = t->global[l];
    const float* cosv = g ? t->cos_g : t->cos_l;
    const float* sinv = g ? t->sin_g : t->sin_l;
    // rotated bf16 hi (kept for the backward) and lo (accurate forward, this forward only) straight from the product
    const int fused = lin_qkv(t, b, T, 3 * H, H, t->n1[l], n1lo, p.qkv, nullptr, cosv, sinv, 2 * H, t->qkv[l],
                              pr ? t->ws_qkvlo : nullptr);
    if (fused != OK && fused != ERR_NOT_SUPPORTED) return fused;
    if (fused == OK) {
    } else if (pr) {   // fp32 qkv → rotated bf16 hi and lo by the prep pass
        RC(lin_fwd(t, T, 3 * H, H, t->n1[l], n1lo, p.qkv, nullptr, bf::EPI_F32, t->ws_qkv32));
        RC(attn_prep(t->ws_qkv32, 1, 3 * H, T, H, t->heads, b->tok_item, b->seg_start, cosv, sinv, t->qkv[l],
                     t->ws_qkvlo, 3 * H, s));
    } else {    // bf16 qkv rotated in place
        RC(lin_fwd(t, T, 3 * H, H, t->n1[l], nullptr, p.qkv, nullptr, bf::EPI_BF16, t->qkv[l]));
        RC(attn_prep(t->qkv[l], 0, 3 * H, T, H, t->heads, b->tok_item, b->seg_start, cosv, sinv, t->qkv[l], nullptr,
                     3 * H, s));
    }
    fa::Args att = attn_args(t, b, t->qkv[l], pr ? t->ws_qkvlo : nullptr, t->heads, g ? -1 : t->window, cosv, sinv,
                             0.f, 0, t->ctx[l], ctxlo, t->lse[l]);
    RC(timed(t, 1, 4.0 * H * (g ? b->pairs_global : b->pairs_local), [&] { return flash_forward(att, b->tiles, s); }));
    LAYA_CUDA(cudaMemcpyAsync(t->X1[l], t->X[l], sizeof(float) * T * H, cudaMemcpyDeviceToDevice, s));
    RC(lin_fwd(t, T, H, H, t->ctx[l], ctxlo, p.wo, nullptr, bf::EPI_F32_ADD, t->X1[l]));
    RC(ln_fwd(ln_args(t, T, t->X1[l], p.n2, NONE, t->eps, t->n2[l], n2lo, nullptr, t->mean2[l], t->rstd2[l]), s));
    if (pr) {
        RC(lin_fwd(t, T, 2 * I, H, t->n2[l], n2lo, p.wi, nullptr, bf::EPI_F32, t->wide32[l]));
        RC(geglu_fwd_f32(t->wide32[l], T, I, t->act[l], actlo, s));
    } else {
        RC(lin_fwd(t, T, 2 * I, H, t->n2[l], nullptr, p.wi, nullptr, bf::EPI_BF16, t->wide[l]));
        RC(geglu_fwd(t->wide[l], T, I, t->act[l], s));
    }
    LAYA_CUDA(cudaMemcpyAsync(t->X[l + 1], t->X1[l], sizeof(float) * T * H, cudaMemcpyDeviceToDevice, s));
    RC(lin_fwd(t, T, H, I, t->act[l], actlo, p.wo2, nullptr, bf::EPI_F32_ADD, t->X[l + 1]));
    return OK;
}

// HeadLayerForward (TrainableDecisionModel.cs:428-468): nn.TransformerEncoderLayer, norm_first, ReLU, dropout on the
// attention probabilities (site 0), the attention output (1), the ReLU output (2) and the feed-forward output (3).
int head_forward(laya_trainer* t, const laya_batch* b, int l) {
    const int T = b->T, H = t->H, FF = t->FF;
    const HeadP& p = t->head[l];
    cudaStream_t s = t->stream;
    const size_t n = static_cast<size_t>(T) * H;
    const bool pr = t->precise;
    bf16 *n1lo = at(t->hn1lo, l), *n2lo = at(t->hn2lo, l), *ctxlo = at(t->hctxlo, l), *actlo = at(t->hactlo, l);
    RC(ln_fwd(ln_args(t, T, t->HIN[l], p.n1w, p.n1b, 1e-5f, t->hn1[l], n1lo, nullptr, t->hm1[l], t->hr1[l]), s));
    if (pr) {   // no rotary in the head: the prep only splits fp32 qkv into hi and lo
        const int fused = lin_qkv(t, b, T, 3 * H, H, t->hn1[l], n1lo, p.inw, t->master + p.inb, nullptr, nullptr, 0,
                                  t->hqkv[l], t->ws_qkvlo);
        if (fused != OK && fused != ERR_NOT_SUPPORTED) return fused;
        if (fused != OK) {
            RC(lin_fwd(t, T, 3 * H, H, t->hn1[l], n1lo, p.inw, t->master + p.inb, bf::EPI_F32, t->ws_qkv32));
            RC(attn_prep(t->ws_qkv32, 1, 3 * H, T, H, t->HH, b->tok_item, b->seg_start, nullptr, nullptr, t->hqkv[l],
                         t->ws_qkvlo, 3 * H, s));
        }
    } else {
        RC(lin_fwd(t, T, 3 * H, H, t->hn1[l], nullptr, p.inw, t->master + p.inb, bf::EPI_BF16, t->hqkv[l]));
    }
    const tr::Mask m0 = head_mask(t, l, 0);
    fa::Args att = attn_args(t, b, t->hqkv[l], pr ? t->ws_qkvlo : nullptr, t->HH, -1, nullptr, nullptr, m0.p, m0.seed,
                             t->hctx[l], ctxlo, t->hlse[l]);
    if (t->masks_pending && m0.p > 0.f) {   // the layer's decisions, drawn at the start of the forward
        LAYA_CUDA(cudaStreamWaitEvent(s, t->mask_done, 0));
        att.dmask = t->dmask + static_cast<size_t>(l) * t->dmask_layer;
        att.dmask_w = t->dmask_w; att.dmask_rows = t->dmask_rows;
    }
    RC(timed(t, 1, 4.0 * H * b->pairs_global, [&] { return flash_forward(att, b->tiles, s); }));
    RC(lin_fwd(t, T, H, H, t->hctx[l], ctxlo, p.outw, t->master + p.outb, bf::EPI_F32, t->R32));
    RC(add_masked(t->HIN[l], t->R32, t->HX1[l], n, head_mask(t, l, 1), s));
    RC(ln_fwd(ln_args(t, T, t->HX1[l], p.n2w, p.n2b, 1e-5f, t->hn2[l], n2lo, nullptr, t->hm2[l], t->hr2[l]), s));
    if (pr) {
        RC(lin_fwd(t, T, FF, H, t->hn2[l], n2lo, p.l1w, t->master + p.l1b, bf::EPI_F32, t->hpre32[l]));
        RC(relu_mask_f32(t->hpre32[l], t->hact[l], actlo, static_cast<size_t>(T) * FF, head_mask(t, l, 2), s));
    } else {
        RC(lin_fwd(t, T, FF, H, t->hn2[l], nullptr, p.l1w, t->master + p.l1b, bf::EPI_BF16, t->hpre[l]));
        RC(relu_mask(t->hpre[l], t->hact[l], static_cast<size_t>(T) * FF, head_mask(t, l, 2), s));
    }
    RC(lin_fwd(t, T, H, FF, t->hact[l], actlo, p.l2w, t->master + p.l2b, bf::EPI_F32, t->R32));
    RC(add_masked(t->HX1[l], t->R32, t->HIN[l + 1], n, head_mask(t, l, 3), s));
    return OK;
}

// TrainableDecisionModel.Forward (TrainableDecisionModel.cs:248-353).
int forward(laya_trainer* t, const laya_batch* b) {
    const int T = b->T, M = b->M, H = t->H;
    cudaStream_t s = t->stream;
    t->masks_pending = false;
    if (t->dmask && t->fwd_training && t->td.head_dropout > 0.f && t->HL > 0) {
        if (!t->mask_stream) {
            LAYA_CUDA(cudaStreamCreateWithFlags(&t->mask_stream, cudaStreamNonBlocking));
            LAYA_CUDA(cudaEventCreateWithFlags(&t->mask_begin, cudaEventDisableTiming));
            LAYA_CUDA(cudaEventCreateWithFlags(&t->mask_done, cudaEventDisableTiming));
        }
        LAYA_CUDA(cudaEventRecord(t->mask_begin, s));
        LAYA_CUDA(cudaStreamWaitEvent(t->mask_stream, t->mask_begin, 0));
        for (int l = 0; l < t->HL; ++l) {
            const tr::Mask m0 = head_mask(t, l, 0);
            fa::Args a = attn_args(t, b, t->hqkv[l], nullptr, t->HH, -1, nullptr, nullptr, m0.p, m0.seed, t->hctx[l],
                                   nullptr, t->hlse[l]);
            uint32_t* mk = t->dmask + static_cast<size_t>(l) * t->dmask_layer;
            a.dmask = mk; a.dmask_w = t->dmask_w; a.dmask_rows = t->dmask_rows;
            RC(drop_mask(a, b->tok_item, mk, t->mask_stream));
        }
        LAYA_CUDA(cudaEventRecord(t->mask_done, t->mask_stream));
        t->masks_pending = true;
    }
    tr::LnFwd e = ln_args(t, T, nullptr, t->emb_norm, NONE, t->eps, nullptr, nullptr, t->X[0], t->emb_mean, t->emb_rstd);
    e.ids = b->ids; e.table = t->master + t->tok_emb; e.vocab = t->V;
    RC(ln_fwd(e, s));
    for (int l = 0; l < t->L; ++l) RC(enc_forward(t, b, l));
    tr::LnFwd f = ln_args(t, T, t->X[t->L], t->final_norm, NONE, t->eps, nullptr, nullptr, t->HIN[0], t->f_mean,
                          t->f_rstd);
    f.temb = t->master + t->type_emb; f.tok_item = b->tok_item; f.qtype = b->qtype;
    RC(ln_fwd(f, s));
    for (int l = 0; l < t->HL; ++l) RC(head_forward(t, b, l));
    // scorer at every option marker: LayerNorm → Linear → GELU → Linear (TrainableDecisionModel.cs:313-331)
    tr::LnFwd sc = ln_args(t, M, t->HIN[t->HL], t->sc0w, t->sc0b, 1e-5f, t->sn16, t->snlo, nullptr, t->smean, t->srstd);
    sc.gather = b->marker_rows;
    RC(ln_fwd(sc, s));
    RC(lin_fwd(t, M, H, H, t->sn16, t->snlo, t->sc1w, t->master + t->sc1b, bf::EPI_F32, t->spre));
    RC(scorer_out(t->spre, M, H, t->master + t->sc3w, t->master + t->sc3b, t->logits, s));
    return OK;
}

// ------------------------------------------------------------------------------------------------ backward
// Gradients at or above element `boundary` of the flat buffer are final: issue the allreduce of every bucket that lies
// entirely there, on the communication stream, after the work enqueued so far.
int grads_ready(laya_trainer* t, size_t boundary) {
    Comm& c = t->comm;
    if (!c.active) return OK;
    bool recorded = false;
    while (c.next < c.buckets.size() && c.buckets[c.next].first >= boundary) {
        if (!recorded) {
            LAYA_CUDA(cudaEventRecord(c.ready, t->stream));
            LAYA_CUDA(cudaStreamWaitEvent(c.stream, c.ready, 0));
            recorded = true;
        }
        const auto& bk = c.buckets[c.next++];
        float* p = t->grad + bk.first;
        ncclResult_t r = g_nccl.allReduce(p, p, bk.second - bk.first, ncclFloat32, ncclSum, c.comm, c.stream);
        if (r != ncclSuccess) return nccl_fail(r, "ncclAllReduce");
    }
    return OK;
}

// HeadLayerBackward (TrainableDecisionModel.cs:605-640); t->dH holds d(output) on entry, d(input) on return.
int head_backward(laya_trainer* t, const laya_batch* b, int l) {
    const int T = b->T, H = t->H, FF = t->FF;
    const HeadP& p = t->head[l];
    cudaStream_t s = t->stream;
    const size_t n = static_cast<size_t>(T) * H;
    float* G = t->grad;
    // out = x1 + drop3(linear2(drop2(relu(linear1(LN2(x1))))))
    RC(cast_mask(t->dH, t->d16, n, head_mask(t, l, 3), s));
    RC(lin_dw(t, T, H, FF, t->d16, t->hact[l], p.l2w));
    RC(colsum_bf16(t->d16, T, H, G + p.l2b, s));
    RC(lin_dx(t, T, H, FF, t->d16, p.l2w, bf::EPI_F32, t->dbig32));
    if (t->precise) RC(relu_mask_bwd_f32(t->dbig32, t->hpre32[l], t->dbig16, static_cast<size_t>(T) * FF, head_mask(t, l, 2), s));
    else RC(relu_mask_bwd(t->dbig32, t->hpre[l], t->dbig16, static_cast<size_t>(T) * FF, head_mask(t, l, 2), s));
    RC(lin_dw(t, T, FF, H, t->dbig16, t->hn2[l], p.l1w));
    RC(colsum_bf16(t->dbig16, T, FF, G + p.l1b, s));
    RC(lin_dx(t, T, FF, H, t->dbig16, p.l1w, bf::EPI_F32, t->dN));
    RC(ln_bwd(lnb_args(t, T, t->HX1[l], t->hm2[l], t->hr2[l], p.n2w, p.n2b, t->dN, t->dH, 1), s));
    // x1 = x + drop1(out_proj(attention(in_proj(LN1(x)))))
    RC(cast_mask(t->dH, t->d16, n, head_mask(t, l, 1), s));
    RC(lin_dw(t, T, H, H, t->d16, t->hctx[l], p.outw));
    RC(colsum_bf16(t->d16, T, H, G + p.outb, s));
    RC(lin_dx(t, T, H, H, t->d16, p.outw, bf::EPI_BF16, t->dctx16));
    const tr::Mask m0 = head_mask(t, l, 0);
    fa::Args att = attn_args(t, b, t->hqkv[l], nullptr, t->HH, -1, nullptr, nullptr, m0.p, m0.seed, t->hctx[l],
                             nullptr, t->hlse[l]);
    if (t->masks_pending && m0.p > 0.f) {   // the decisions the forward drew
        att.dmask = t->dmask + static_cast<size_t>(l) * t->dmask_layer;
        att.dmask_w = t->dmask_w; att.dmask_rows = t->dmask_rows;
    }
    RC(timed(t, 2, 8.0 * H * b->pairs_global, [&] { return flash_backward(att, b->tiles, T, s); }));
    RC(lin_dw(t, T, 3 * H, H, t->dqkv16, t->hn1[l], p.inw));
    RC(colsum_bf16(t->dqkv16, T, 3 * H, G + p.inb, s));
    RC(lin_dx(t, T, 3 * H, H, t->dqkv16, p.inw, bf::EPI_F32, t->dN));
    RC(ln_bwd(lnb_args(t, T, t->HIN[l], t->hm1[l], t->hr1[l], p.n1w, p.n1b, t->dN, t->dH, 1), s));
    return OK;
}

// EncoderLayerBackward (TrainableDecisionModel.cs:551-603); t->dH holds d(output) on entry, d(input) on return.
int enc_backward(laya_trainer* t, const laya_batch* b, int l, bool need_dx) {
    const int T = b->T, H = t->H, I = t->I;
    const EncP& p = t->enc[l];
    cudaStream_t s = t->stream;
    const size_t n = static_cast<size_t>(T) * H;
    // x2 = x1 + Wo2 · (gelu(u) ⊙ gate), [u | gate] = Wi · LN2(x1)
    RC(f32_to_bf16(t->dH, t->d16, n, s));
    RC(lin_dw(t, T, H, I, t->d16, t->act[l], p.wo2));
    RC(lin_dx(t, T, H, I, t->d16, p.wo2, bf::EPI_F32, t->dbig32));
    if (t->precise) RC(geglu_bwd_f32(t->wide32[l], t->dbig32, T, I, t->dbig16, s));
    else RC(geglu_bwd(t->wide[l], t->dbig32, T, I, t->dbig16, s));
    RC(lin_dw(t, T, 2 * I, H, t->dbig16, t->n2[l], p.wi));
    RC(lin_dx(t, T, 2 * I, H, t->dbig16, p.wi, bf::EPI_F32, t->dN));
    RC(ln_bwd(lnb_args(t, T, t->X1[l], t->mean2[l], t->rstd2[l], p.n2, NONE, t->dN, t->dH, 1), s));
    // x1 = x + Wo · attention(Wqkv · LN1(x))
    RC(f32_to_bf16(t->dH, t->d16, n, s));
    RC(lin_dw(t, T, H, H, t->d16, t->ctx[l], p.wo));
    RC(lin_dx(t, T, H, H, t->d16, p.wo, bf::EPI_BF16, t->dctx16));
    const bool g = t->global[l];
    fa::Args att = attn_args(t, b, t->qkv[l], nullptr, t->heads, g ? -1 : t->window, g ? t->cos_g : t->cos_l,
                             g ? t->sin_g : t->sin_l, 0.f, 0, t->ctx[l], nullptr, t->lse[l]);
    RC(timed(t, 2, 8.0 * H * (g ? b->pairs_global : b->pairs_local), [&] { return flash_backward(att, b->tiles, T, s); }));
    RC(lin_dw(t, T, 3 * H, H, t->dqkv16, t->n1[l], p.qkv));
    if (p.n1 == NONE) {
        // identity norm: dx += dqkv · Wqkv
        if (need_dx) RC(lin_dx(t, T, 3 * H, H, t->dqkv16, p.qkv, bf::EPI_F32_ADD, t->dH));
    } else {
        // the norm's γ trains even when nothing below needs dx
        RC(lin_dx(t, T, 3 * H, H, t->dqkv16, p.qkv, bf::EPI_F32, t->dN));
        RC(ln_bwd(lnb_args(t, T, t->X[l], t->mean1[l], t->rstd1[l], p.n1, NONE, t->dN, need_dx ? t->dH : nullptr, 1), s));
    }
    return OK;
}

// TrainableDecisionModel.Backward (TrainableDecisionModel.cs:479-549).
int backward(laya_trainer* t, const laya_batch* b) {
    const int T = b->T, M = b->M, H = t->H;
    cudaStream_t s = t->stream;
    float* G = t->grad;
    LAYA_CUDA(cudaMemsetAsync(t->dH, 0, sizeof(float) * T * H, s));
    RC(scorer_bwd(t->spre, t->dlog, M, H, t->master + t->sc3w, t->dpre16, G + t->sc1b, G + t->sc3w, G + t->sc3b, s));
    RC(lin_dx(t, M, H, H, t->dpre16, t->sc1w, bf::EPI_F32, t->dsn));
    RC(lin_dw(t, M, H, H, t->dpre16, t->sn16, t->sc1w));
    tr::LnBwd sb = lnb_args(t, M, t->HIN[t->HL], t->smean, t->srstd, t->sc0w, t->sc0b, t->dsn, t->dH, 1);
    sb.gather = b->marker_rows;
    sb.scatter = b->marker_rows;
    RC(ln_bwd(sb, s));
    RC(grads_ready(t, t->scorer_start));
    for (int l = t->HL - 1; l >= 0; --l) {
        RC(head_backward(t, b, l));
        RC(grads_ready(t, t->head_start[l]));
    }
    RC(type_grad(t->dH, b->tok_item, b->qtype, T, H, G + t->type_emb, s));
    RC(grads_ready(t, t->type_emb));
    if (t->first_trainable < t->L) {
        RC(ln_bwd(lnb_args(t, T, t->X[t->L], t->f_mean, t->f_rstd, t->final_norm, NONE, t->dH, t->dH, 0), s));
        RC(grads_ready(t, t->final_norm));
        for (int l = t->L - 1; l >= t->first_trainable; --l) {
            RC(enc_backward(t, b, l, l > t->first_trainable || t->emb_trainable));
            RC(grads_ready(t, t->enc[l].n1 == NONE ? t->enc[l].qkv : t->enc[l].n1));
        }
        if (t->emb_trainable && t->first_trainable == 0) {
            tr::LnBwd eb = lnb_args(t, T, t->master + t->tok_emb, t->emb_mean, t->emb_rstd, t->emb_norm, NONE, t->dH,
                                    t->dH, 0);
            eb.gather = b->ids;
            RC(ln_bwd(eb, s));
            RC(scatter_rows(t->dH, b->ids, T, H, G + t->tok_emb, s));
        }
    }
    RC(grads_ready(t, 0));
    return OK;
}

int reduce_all(laya_trainer* t) {
    Comm& c = t->comm;
    c.active = true;
    c.next = 0;
    RC(grads_ready(t, 0));
    c.active = false;
    return OK;
}

}  // namespace
}  // namespace laya

using namespace laya;

// ================================================================================================ C ABI
extern "C" {

int laya_trainer_create(const laya_model_desc* desc, const laya_train_desc* train, int device, laya_trainer** out) {
    if (!desc || !train || !out) { set_error("null argument"); return ERR_ARGUMENT; }
    *out = nullptr;
    const laya_model_desc& d = *desc;
    if (d.hidden <= 0 || d.heads <= 0 || d.hidden % d.heads || (d.hidden / d.heads != 64 && d.hidden / d.heads != 32) ||
        d.hidden % 64 || d.hidden > 1024 || d.layers < 0 || d.vocab <= 0 || d.intermediate <= 0 || d.intermediate % 8 ||
        d.max_tokens <= 0 || d.max_items <= 0 || d.max_markers <= 0 || d.head_layers < 0) {
        set_error("invalid training geometry (hidden a multiple of 64 up to 1024, head_dim 32 or 64, "
                  "intermediate a multiple of 8)");
        return ERR_ARGUMENT;
    }
    if (train->head_dropout < 0.f || train->head_dropout >= 1.f) { set_error("head_dropout must be in [0, 1)"); return ERR_ARGUMENT; }
    int ndev = 0;
    LAYA_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) { set_error("no such CUDA device"); return ERR_ARGUMENT; }
    cudaDeviceProp prop;
    LAYA_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) {
        set_error("laya_b200 kernels are built for sm_100a (B200)");
        return ERR_NOT_SUPPORTED;
    }
    DeviceGuard g(device);
    laya_trainer* t = new laya_trainer();
    t->device = device;
    t->d = d;
    t->d.layer_kinds = nullptr;
    t->td = *train;
    if (t->d.act_hidden <= 0) t->d.act_hidden = 256;
    if (t->d.n_act <= 0) t->d.n_act = 2;
    if (t->d.global_every <= 0) t->d.global_every = 3;
    t->H = d.hidden; t->I = d.intermediate; t->L = d.layers; t->heads = d.heads; t->hd = d.hidden / d.heads;
    t->HL = d.head_layers; t->HH = std::max(1, d.hidden / 64); t->FF = 4 * d.hidden; t->V = d.vocab;
    t->window = d.local_attention / 2;
    t->eps = d.norm_eps > 0 ? d.norm_eps : 1e-5f;
    t->global.resize(t->L);
    for (int i = 0; i < t->L; ++i) t->global[i] = d.layer_kinds ? (d.layer_kinds[i] != 0) : (i % t->d.global_every == 0);
    t->lr[0] = train->encoder_lr; t->lr[1] = train->head_lr;
    if (train->forward_mode != LAYA_FORWARD_ACCURATE && train->forward_mode != LAYA_FORWARD_BF16) {
        delete t;
        set_error("unknown forward_mode");
        return ERR_ARGUMENT;
    }
    t->precise = train->forward_mode == LAYA_FORWARD_ACCURATE;
    t->maxpos = train->max_segment > 0 ? train->max_segment : std::min(d.max_tokens, 8192);
    if (t->maxpos > (1 << 21)) { delete t; set_error("max_segment above 2^21"); return ERR_ARGUMENT; }
    auto fail = [&](int rc) { laya_trainer_destroy(t); return rc; };
    if (cudaStreamCreateWithFlags(&t->own, cudaStreamNonBlocking) != cudaSuccess)
        return fail(cuda_fail(cudaGetLastError(), "cudaStreamCreate"));
    t->stream = t->own;

    build_registry(t);
    int rc;
    const size_t P = t->P;
    if ((rc = dalloc_t(t, &t->master, P)) || (rc = dalloc_t(t, &t->grad, P)) || (rc = dalloc_t(t, &t->m, P)) ||
        (rc = dalloc_t(t, &t->v, P)) || (rc = dalloc_t(t, &t->shadow, P)) || (rc = dalloc_t(t, &t->err, 1)) ||
        (rc = dalloc_t(t, &t->red, 8 + SUMSQ_BLOCKS)))
        return fail(rc);
    if (t->precise) {
        if ((rc = dalloc_t(t, &t->shadow_lo, P))) return fail(rc);
        cudaMemsetAsync(t->shadow_lo, 0, sizeof(bf16) * P, t->stream);
    }
    cudaMemsetAsync(t->master, 0, sizeof(float) * P, t->stream);
    cudaMemsetAsync(t->grad, 0, sizeof(float) * P, t->stream);
    cudaMemsetAsync(t->m, 0, sizeof(float) * P, t->stream);
    cudaMemsetAsync(t->v, 0, sizeof(float) * P, t->stream);
    cudaMemsetAsync(t->shadow, 0, sizeof(bf16) * P, t->stream);
    cudaMemsetAsync(t->err, 0, sizeof(int), t->stream);
    cudaMemsetAsync(t->red, 0, sizeof(double) * 8, t->stream);
    if (cudaMallocHost(&t->h_red, sizeof(double) * 8) != cudaSuccess) return fail(cuda_fail(cudaGetLastError(), "cudaMallocHost"));

    // tape and workspace
    const int H = t->H, I = t->I, L = t->L, HL = t->HL, FF = t->FF;
    t->Tc = d.max_tokens; t->Mc = d.max_markers; t->Nc = d.max_items;
    t->tiles_cap = d.max_tokens / 64 + d.max_items + 1;
    const size_t T = t->Tc, M = t->Mc;
    t->X.resize(L + 1); t->X1.resize(L); t->mean1.resize(L); t->rstd1.resize(L); t->mean2.resize(L); t->rstd2.resize(L);
    t->lse.resize(L); t->n1.resize(L); t->qkv.resize(L); t->ctx.resize(L); t->n2.resize(L); t->wide.resize(L);
    t->act.resize(L);
    for (int l = 0; l <= L; ++l)
        if ((rc = dalloc_t(t, &t->X[l], T * H))) return fail(rc);
    const bool pr = t->precise;
    if (pr) {
        t->n1lo.resize(L); t->ctxlo.resize(L); t->n2lo.resize(L); t->actlo.resize(L); t->wide32.resize(L);
        if ((rc = dalloc_t(t, &t->ws_qkv32, T * 3 * H)) || (rc = dalloc_t(t, &t->ws_qkvlo, T * 3 * H))) return fail(rc);
    } else {
        t->wide.resize(L);
    }
    for (int l = 0; l < L; ++l) {
        if ((rc = dalloc_t(t, &t->X1[l], T * H)) || (rc = dalloc_t(t, &t->mean1[l], T)) ||
            (rc = dalloc_t(t, &t->rstd1[l], T)) || (rc = dalloc_t(t, &t->mean2[l], T)) ||
            (rc = dalloc_t(t, &t->rstd2[l], T)) || (rc = dalloc_t(t, &t->lse[l], T * t->heads)) ||
            (rc = dalloc_t(t, &t->n1[l], T * H)) || (rc = dalloc_t(t, &t->ctx[l], T * H)) ||
            (rc = dalloc_t(t, &t->n2[l], T * H)) || (rc = dalloc_t(t, &t->act[l], T * I)) ||
            (rc = dalloc_t(t, &t->qkv[l], T * 3 * H)))
            return fail(rc);
        if (pr) {
            if ((rc = dalloc_t(t, &t->n1lo[l], T * H)) || (rc = dalloc_t(t, &t->ctxlo[l], T * H)) ||
                (rc = dalloc_t(t, &t->n2lo[l], T * H)) || (rc = dalloc_t(t, &t->actlo[l], T * I)) ||
                (rc = dalloc_t(t, &t->wide32[l], T * 2 * I)))
                return fail(rc);
        } else if ((rc = dalloc_t(t, &t->wide[l], T * 2 * I))) {
            return fail(rc);
        }
    }
    if ((rc = dalloc_t(t, &t->emb_mean, T)) || (rc = dalloc_t(t, &t->emb_rstd, T)) || (rc = dalloc_t(t, &t->f_mean, T)) ||
        (rc = dalloc_t(t, &t->f_rstd, T)))
        return fail(rc);
    t->HIN.resize(HL + 1); t->HX1.resize(HL); t->hm1.resize(HL); t->hr1.resize(HL); t->hm2.resize(HL); t->hr2.resize(HL);
    t->hlse.resize(HL); t->hn1.resize(HL); t->hctx.resize(HL); t->hn2.resize(HL); t->hact.resize(HL); t->hqkv.resize(HL);
    if (pr) {
        t->hn1lo.resize(HL); t->hctxlo.resize(HL); t->hn2lo.resize(HL); t->hactlo.resize(HL); t->hpre32.resize(HL);
    } else {
        t->hpre.resize(HL);
    }
    for (int l = 0; l <= HL; ++l)
        if ((rc = dalloc_t(t, &t->HIN[l], T * H))) return fail(rc);
    for (int l = 0; l < HL; ++l) {
        if ((rc = dalloc_t(t, &t->HX1[l], T * H)) || (rc = dalloc_t(t, &t->hm1[l], T)) || (rc = dalloc_t(t, &t->hr1[l], T)) ||
            (rc = dalloc_t(t, &t->hm2[l], T)) || (rc = dalloc_t(t, &t->hr2[l], T)) ||
            (rc = dalloc_t(t, &t->hlse[l], T * t->HH)) || (rc = dalloc_t(t, &t->hn1[l], T * H)) ||
            (rc = dalloc_t(t, &t->hctx[l], T * H)) || (rc = dalloc_t(t, &t->hn2[l], T * H)) ||
            (rc = dalloc_t(t, &t->hact[l], T * FF)) || (rc = dalloc_t(t, &t->hqkv[l], T * 3 * H)))
            return fail(rc);
        if (pr) {
            if ((rc = dalloc_t(t, &t->hn1lo[l], T * H)) || (rc = dalloc_t(t, &t->hctxlo[l], T * H)) ||
                (rc = dalloc_t(t, &t->hn2lo[l], T * H)) || (rc = dalloc_t(t, &t->hactlo[l], T * FF)) ||
                (rc = dalloc_t(t, &t->hpre32[l], T * FF)))
                return fail(rc);
        } else if ((rc = dalloc_t(t, &t->hpre[l], T * FF))) {
            return fail(rc);
        }
    }
    const size_t big = std::max<size_t>(2 * I, FF);
    if (pr && (rc = dalloc_t(t, &t->snlo, M * H))) return fail(rc);
    if ((rc = dalloc_t(t, &t->sn16, M * H)) || (rc = dalloc_t(t, &t->smean, M)) || (rc = dalloc_t(t, &t->srstd, M)) ||
        (rc = dalloc_t(t, &t->spre, M * H)) || (rc = dalloc_t(t, &t->logits, M)) || (rc = dalloc_t(t, &t->dlog, M)) ||
        (rc = dalloc_t(t, &t->R32, T * H)) || (rc = dalloc_t(t, &t->dH, T * H)) || (rc = dalloc_t(t, &t->dN, T * H)) ||
        (rc = dalloc_t(t, &t->dbig32, T * big)) || (rc = dalloc_t(t, &t->dsum, T * std::max(t->heads, t->HH))) ||
        (rc = dalloc_t(t, &t->dsn, M * H)) || (rc = dalloc_t(t, &t->d16, T * H)) || (rc = dalloc_t(t, &t->dctx16, T * H)) ||
        (rc = dalloc_t(t, &t->dqkv16, T * 3 * H)) || (rc = dalloc_t(t, &t->dbig16, T * big)) ||
        (rc = dalloc_t(t, &t->dpre16, M * H)))
        return fail(rc);
    if ((rc = dalloc(t, reinterpret_cast<void**>(&t->rl_scratch), rlcd_scratch_bytes(MAX_GROUPS, t->Nc, t->Mc))))
        return fail(rc);
    {   // the attention backward's dS scratch: per 128-row tile of the batch, ceil(max segment / 64) query tiles of
        // 16 KB per head, after one zero tile; long-context geometries that would need more than DS_SCRATCH_MAX
        // recompute S and dP in the dQ kernel instead
        const int heads = std::max(t->heads, t->HH);
        const size_t tiles = static_cast<size_t>(d.max_tokens + 127) / 128 + static_cast<size_t>(d.max_items);
        const int nq = (t->maxpos + 63) / 64;
        const size_t bytes = (1 + tiles * nq * heads) * 16384;
        if (t->hd == 64 && bytes <= DS_SCRATCH_MAX) {
            if ((rc = dalloc(t, reinterpret_cast<void**>(&t->ds), bytes))) return fail(rc);
            if (cudaMemset(t->ds, 0, 16384) != cudaSuccess) return fail(cuda_fail(cudaGetLastError(), "dS zero tile"));
            t->ds_nq = nq;
        }
    }
    if (t->HL > 0) {   // the head layers' dropout decisions: [layer][head][row][4 words per 128 keys of the segment]
        const int w = 4 * ((t->maxpos + 127) / 128);
        const size_t words = static_cast<size_t>(t->HH) * static_cast<size_t>(d.max_tokens) * static_cast<size_t>(w);
        if (words * t->HL * 4 <= DMASK_MAX) {
            if ((rc = dalloc_t(t, &t->dmask, words * t->HL))) return fail(rc);
            t->dmask_w = w;
            t->dmask_rows = d.max_tokens;
            t->dmask_layer = words;
        }
    }
    {   // the LayerNorm backward's per-CTA dγ/dβ partials
        int nsm = 0;
        if ((rc = sm_count(t->device, &nsm))) return fail(rc);
        if ((rc = dalloc_t(t, &t->ln_part, static_cast<size_t>(nsm) * tr::LN_PART_CTAS_PER_SM * 2 * H))) return fail(rc);
    }

    // Rotary tables (Rotary, Ops.cs:446-480): angles in double, stored fp32, [position, head_dim/2].
    const int half = t->hd / 2;
    std::vector<float> cg(static_cast<size_t>(t->maxpos) * half), sg(cg.size()), cl(cg.size()), sl(cg.size());
    for (int i = 0; i < half; ++i) {
        const double ig = 1.0 / std::pow(d.theta_global, 2.0 * i / t->hd);
        const double il = 1.0 / std::pow(d.theta_local, 2.0 * i / t->hd);
        for (int p = 0; p < t->maxpos; ++p) {
            cg[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(p * ig));
            sg[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(p * ig));
            cl[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(p * il));
            sl[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(p * il));
        }
    }
    if ((rc = dalloc_t(t, &t->cos_g, cg.size())) || (rc = dalloc_t(t, &t->sin_g, cg.size())) ||
        (rc = dalloc_t(t, &t->cos_l, cg.size())) || (rc = dalloc_t(t, &t->sin_l, cg.size())))
        return fail(rc);
    cudaMemcpyAsync(t->cos_g, cg.data(), sizeof(float) * cg.size(), cudaMemcpyHostToDevice, t->stream);
    cudaMemcpyAsync(t->sin_g, sg.data(), sizeof(float) * cg.size(), cudaMemcpyHostToDevice, t->stream);
    cudaMemcpyAsync(t->cos_l, cl.data(), sizeof(float) * cg.size(), cudaMemcpyHostToDevice, t->stream);
    cudaMemcpyAsync(t->sin_l, sl.data(), sizeof(float) * cg.size(), cudaMemcpyHostToDevice, t->stream);
    if (cudaStreamSynchronize(t->stream) != cudaSuccess) return fail(cuda_fail(cudaGetLastError(), "trainer setup"));
    *out = t;
    return OK;
}

int laya_trainer_destroy(laya_trainer* t) {
    if (!t) return OK;
    DeviceGuard g(t->device);
    if (t->stream) cudaStreamSynchronize(t->stream);
    if (t->comm.stream) cudaStreamSynchronize(t->comm.stream);
    if (t->comm.comm && g_nccl.commDestroy) g_nccl.commDestroy(t->comm.comm);
    if (t->comm.ready) cudaEventDestroy(t->comm.ready);
    if (t->comm.done) cudaEventDestroy(t->comm.done);
    if (t->comm.stream) cudaStreamDestroy(t->comm.stream);
    if (t->mask_stream) { cudaStreamSynchronize(t->mask_stream); cudaStreamDestroy(t->mask_stream); }
    if (t->mask_begin) cudaEventDestroy(t->mask_begin);
    if (t->mask_done) cudaEventDestroy(t->mask_done);
    for (void* p : t->allocs) cudaFree(p);
    for (auto& e : t->ev_pool) { cudaEventDestroy(e.first); cudaEventDestroy(e.second); }
    if (t->h_red) cudaFreeHost(t->h_red);
    if (t->own) cudaStreamDestroy(t->own);
    delete t;
    return OK;
}

int laya_trainer_set_stream(laya_trainer* t, void* stream) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    t->stream = static_cast<cudaStream_t>(stream);
    return OK;
}
int laya_trainer_get_stream(laya_trainer* t, void** stream) {
    if (!t || !stream) { set_error("null argument"); return ERR_ARGUMENT; }
    *stream = static_cast<void*>(t->stream);
    return OK;
}
int laya_trainer_synchronize(laya_trainer* t) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    if (t->comm.stream) LAYA_CUDA(cudaStreamSynchronize(t->comm.stream));
    LAYA_CUDA(cudaStreamSynchronize(t->stream));
    return check_device_error(t);
}

static int find_param(laya_trainer* t, const char* name, const Param** p) {
    if (!t || !name) { set_error("null argument"); return ERR_ARGUMENT; }
    auto it = t->index.find(name);
    if (it == t->index.end()) { set_error(std::string("no trainable tensor named ") + name); return ERR_NOT_FOUND; }
    *p = &t->params[it->second];
    return OK;
}

int laya_trainer_upload(laya_trainer* t, const char* name, int dtype, const int64_t* shape, int rank, const void* host) {
    if (!t || !name || !host || (rank > 0 && !shape)) { set_error("null argument"); return ERR_ARGUMENT; }
    if (std::strcmp(name, "temperature") == 0) return OK;   // calibration state, not a trained parameter
    const Param* p;
    RC(find_param(t, name, &p));
    int64_t count = 1;
    for (int i = 0; i < rank; ++i) count *= shape[i];
    const int64_t n = p->rows * p->cols;
    const bool shape_ok = count == n && (rank == 1 ? (p->rows == 1 || p->cols == 1)
                                                   : rank == 2 && shape[0] == p->rows && shape[1] == p->cols);
    if (!shape_ok) { set_error(std::string("shape mismatch for ") + name); return ERR_ARGUMENT; }
    std::vector<float> buf(n);
    if (dtype == LAYA_F32) {
        std::memcpy(buf.data(), host, sizeof(float) * n);
    } else if (dtype == LAYA_BF16) {
        const uint16_t* h = static_cast<const uint16_t*>(host);
        for (int64_t i = 0; i < n; ++i) {
            const uint32_t u = static_cast<uint32_t>(h[i]) << 16;
            std::memcpy(&buf[i], &u, 4);
        }
    } else if (dtype == LAYA_F16) {
        const __half* h = static_cast<const __half*>(host);
        for (int64_t i = 0; i < n; ++i) buf[i] = __half2float(h[i]);
    } else {
        set_error("trainer tensors are uploaded as F32, BF16 or F16");
        return ERR_ARGUMENT;
    }
    DeviceGuard g(t->device);
    LAYA_CUDA(cudaMemcpyAsync(t->master + p->off, buf.data(), sizeof(float) * n, cudaMemcpyHostToDevice, t->stream));
    RC(f32_split_bf16(t->master + p->off, t->shadow + p->off, t->shadow_lo ? t->shadow_lo + p->off : nullptr,
                      static_cast<size_t>(n), t->stream));
    LAYA_CUDA(cudaStreamSynchronize(t->stream));
    Param& q = t->params[t->index[name]];
    q.shape.assign(shape, shape + rank);
    q.stored = dtype;
    return OK;
}

static int download_range(laya_trainer* t, const char* name, const float* base, float* host, int64_t count) {
    const Param* p;
    RC(find_param(t, name, &p));
    if (!host || count != p->rows * p->cols) { set_error(std::string("count mismatch for ") + name); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    if (t->comm.stream) LAYA_CUDA(cudaStreamSynchronize(t->comm.stream));
    LAYA_CUDA(cudaMemcpyAsync(host, base + p->off, sizeof(float) * count, cudaMemcpyDeviceToHost, t->stream));
    LAYA_CUDA(cudaStreamSynchronize(t->stream));
    return OK;
}
int laya_trainer_download(laya_trainer* t, const char* name, float* host, int64_t count) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    return download_range(t, name, t->master, host, count);
}
int laya_trainer_download_grad(laya_trainer* t, const char* name, float* host, int64_t count) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    return download_range(t, name, t->grad, host, count);
}

// ------------------------------------------------------------------------------------------------ calibration
namespace {
struct CalSample {
    int qtype;
    const float* logits;
    const float* target;
    int k;
};
const char* kTypeNames[3] = {"choice", "score", "noul"};

// TemperatureFitting.FitOne (TemperatureFitting.cs:36-72): the temperature minimising the mean soft cross-entropy,
// golden-section search over log T in double, samples in order; fewer than 10 samples give 1.
float fit_one(const std::vector<const CalSample*>& ss) {
    if (ss.size() < 10) return 1.0f;
    auto objective = [&](double log_t) {
        const double t = std::exp(log_t);
        double total = 0.0;
        for (const CalSample* sp : ss) {
            double mx = -INFINITY;
            for (int i = 0; i < sp->k; ++i) mx = std::max(mx, sp->logits[i] / t);
            double sum = 0.0;
            for (int i = 0; i < sp->k; ++i) sum += std::exp(sp->logits[i] / t - mx);
            const double log_sum = mx + std::log(sum);
            for (int i = 0; i < sp->k; ++i) total -= sp->target[i] * (sp->logits[i] / t - log_sum);
        }
        return total / static_cast<double>(ss.size());
    };
    double low = std::log(0.02), high = std::log(50.0);
    const double ratio = (std::sqrt(5.0) - 1) / 2;
    double a = high - ratio * (high - low), b = low + ratio * (high - low);
    double fa = objective(a), fb = objective(b);
    for (int it = 0; it < 80 && high - low > 1e-7; ++it) {
        if (fa < fb) {
            high = b; b = a; fb = fa;
            a = high - ratio * (high - low);
            fa = objective(a);
        } else {
            low = a; a = b; fa = fb;
            b = low + ratio * (high - low);
            fb = objective(b);
        }
    }
    return static_cast<float>(std::exp((low + high) / 2));
}
// Calibration.ClampTemperature (Laya/Runtime/Calibration.cs:23-24).
float clamp_temperature(float t) { return std::isfinite(t) ? std::min(std::max(t, 0.5f), 5.0f) : 1.0f; }

// TemperatureFitting.Fit (TemperatureFitting.cs:78-101).
int fit_temperatures(const std::vector<CalSample>& samples, int min_bucket, laya_temperature_fit* out) {
    std::memset(out, 0, sizeof *out);
    for (int q = 0; q < 3; ++q) {
        std::vector<const CalSample*> sel;
        for (const CalSample& sp : samples)
            if (sp.qtype == q) sel.push_back(&sp);
        out->by_type[q] = sel.empty() ? 1.2f : clamp_temperature(fit_one(sel));
    }
    std::vector<std::string> keys;
    std::vector<std::vector<const CalSample*>> groups;
    for (const CalSample& sp : samples) {
        const int k = sp.k;
        const std::string key = std::string(kTypeNames[sp.qtype == 0 ? 0 : sp.qtype == 1 ? 1 : 2]) + ":" +
                                (k <= 2 ? "2" : k <= 5 ? "3-5" : k <= 10 ? "6-10" : "11+");
        size_t g = 0;
        while (g < keys.size() && keys[g] != key) ++g;
        if (g == keys.size()) {
            if (keys.size() == LAYA_MAX_TEMPERATURE_BUCKETS) { set_error("more temperature buckets than the fit holds"); return ERR_ARGUMENT; }
            keys.push_back(key);
            groups.emplace_back();
        }
        groups[g].push_back(&sp);
    }
    out->n_buckets = static_cast<int>(keys.size());
    for (size_t g = 0; g < keys.size(); ++g) {
        std::snprintf(out->bucket[g], sizeof out->bucket[g], "%s", keys[g].c_str());
        out->bucket_count[g] = static_cast<int>(groups[g].size());
        out->bucket_fitted[g] = static_cast<int>(groups[g].size()) >= min_bucket;
        out->bucket_temperature[g] = out->bucket_fitted[g] ? clamp_temperature(fit_one(groups[g])) : 1.0f;
    }
    return OK;
}
}  // namespace

int laya_fit_temperatures(const int32_t* qtype, const int32_t* options, const float* logits, const float* targets,
                          int n, int min_bucket_samples, laya_temperature_fit* out) {
    if (!out || n < 0 || (n > 0 && (!qtype || !options || !logits || !targets))) { set_error("invalid argument"); return ERR_ARGUMENT; }
    std::vector<CalSample> samples;
    size_t off = 0;
    for (int i = 0; i < n; ++i) {
        if (options[i] <= 0) { set_error("every sample needs at least one option"); return ERR_ARGUMENT; }
        samples.push_back({qtype[i], logits + off, targets + off, options[i]});
        off += static_cast<size_t>(options[i]);
    }
    return fit_temperatures(samples, min_bucket_samples, out);
}

// Trainer.Calibrate (Laya.Training/Trainer.cs:200-211): forward-only passes (no dropout) over the calibration
// batches on the device, then TemperatureFitting.Fit on their option logits and soft targets.
int laya_train_calibrate(laya_trainer* t, laya_batch* const* batches, int n_batches, int min_bucket_samples,
                         laya_temperature_fit* out) {
    if (!t || !out || n_batches < 0 || (n_batches > 0 && !batches)) { set_error("invalid argument"); return ERR_ARGUMENT; }
    std::vector<std::vector<float>> logits(n_batches), targets(n_batches);
    std::vector<CalSample> samples;
    for (int bi = 0; bi < n_batches; ++bi) {
        laya_batch* b = batches[bi];
        if (!b || b->owner != t) { set_error("batch does not belong to this trainer"); return ERR_ARGUMENT; }
        logits[bi].resize(std::max(b->M, 1));
        RC(laya_train_forward(t, b, 0, 0, logits[bi].data()));
        // the batch's staged host copy holds its question types, option counts and targets
        const char* h = static_cast<const char*>(b->host);
        const int32_t* qt = reinterpret_cast<const int32_t*>(h + b->o_qtype);
        const int32_t* mc = reinterpret_cast<const int32_t*>(h + b->o_mk_count);
        const float* tg = reinterpret_cast<const float*>(h + b->o_targets);
        targets[bi].assign(tg, tg + b->M);
        size_t off = 0;
        for (int i = 0; i < b->n; ++i) {
            samples.push_back({qt[i], logits[bi].data() + off, targets[bi].data() + off, mc[i]});
            off += static_cast<size_t>(mc[i]);
        }
    }
    return fit_temperatures(samples, min_bucket_samples, out);
}

// ------------------------------------------------------------------------------------------------ checkpoints
// TrainableDecisionModel.Save's model.safetensors (TrainableDecisionModel.cs:649-661 through SafetensorsWriter,
// Base/Io/SafetensorsWriter.cs:17-64): every parameter under its name, in the dtype it was loaded in, written to
// path + ".tmp" and moved over path.  With the optimizer: AdamW's m and v as F32 "optimizer.m.<name>" /
// "optimizer.v.<name>" and the step count in the metadata, so that a restore resumes the same trajectory (state the
// reference does not save).
int laya_trainer_save_checkpoint(laya_trainer* t, const char* path, int with_optimizer) {
    if (!t || !path) { set_error("null argument"); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    if (t->comm.stream) LAYA_CUDA(cudaStreamSynchronize(t->comm.stream));
    std::vector<float> master(t->P), m, v;
    LAYA_CUDA(cudaMemcpyAsync(master.data(), t->master, sizeof(float) * t->P, cudaMemcpyDeviceToHost, t->stream));
    if (with_optimizer) {
        m.resize(t->P);
        v.resize(t->P);
        LAYA_CUDA(cudaMemcpyAsync(m.data(), t->m, sizeof(float) * t->P, cudaMemcpyDeviceToHost, t->stream));
        LAYA_CUDA(cudaMemcpyAsync(v.data(), t->v, sizeof(float) * t->P, cudaMemcpyDeviceToHost, t->stream));
    }
    LAYA_CUDA(cudaStreamSynchronize(t->stream));
    struct Out { std::string name, dtype; const std::vector<int64_t>* shape; const float* data; size_t n; };
    std::vector<Out> outs;
    for (const Param& p : t->params) {
        const int st = p.stored;
        outs.push_back({p.name, st == LAYA_BF16 ? "BF16" : st == LAYA_F16 ? "F16" : "F32", &p.shape,
                        master.data() + p.off, static_cast<size_t>(p.rows * p.cols)});
    }
    if (with_optimizer)
        for (const Param& p : t->params) {
            outs.push_back({"optimizer.m." + p.name, "F32", &p.shape, m.data() + p.off, static_cast<size_t>(p.rows * p.cols)});
            outs.push_back({"optimizer.v." + p.name, "F32", &p.shape, v.data() + p.off, static_cast<size_t>(p.rows * p.cols)});
        }
    std::string js = "{";
    if (with_optimizer)
        js += "\"__metadata__\":{\"format\":\"laya_b200\",\"optimizer_step\":\"" + std::to_string(t->steps) + "\"},";
    uint64_t off = 0;
    for (size_t i = 0; i < outs.size(); ++i) {
        const uint64_t bytes = outs[i].n * st::elem_size(outs[i].dtype);
        js += "\"" + st::escape(outs[i].name) + "\":{\"dtype\":\"" + outs[i].dtype + "\",\"shape\":[";
        for (size_t k = 0; k < outs[i].shape->size(); ++k) js += (k ? "," : "") + std::to_string((*outs[i].shape)[k]);
        js += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + bytes) + "]}";
        js += i + 1 < outs.size() ? "," : "";
        off += bytes;
    }
    js += "}";
    while (js.size() % 8) js += ' ';
    const std::string tmp = std::string(path) + ".tmp";
    std::FILE* f = std::fopen(tmp.c_str(), "wb");
    if (!f) { set_error(std::string("cannot create ") + tmp); return ERR_ARGUMENT; }
    unsigned char len[8];
    for (int i = 0; i < 8; ++i) len[i] = static_cast<unsigned char>((static_cast<uint64_t>(js.size()) >> (8 * i)) & 0xFF);
    bool ok = std::fwrite(len, 1, 8, f) == 8 && std::fwrite(js.data(), 1, js.size(), f) == js.size();
    std::vector<uint16_t> half;
    for (const Out& o : outs) {
        if (!ok) break;
        if (o.dtype == "F32") {
            ok = std::fwrite(o.data, sizeof(float), o.n, f) == o.n;
        } else {
            half.resize(o.n);
            for (size_t i = 0; i < o.n; ++i) {
                if (o.dtype == "BF16") half[i] = st::to_bf16(o.data[i]);
                else {
                    const __half hv = __float2half_rn(o.data[i]);   // (Half)value: round to nearest even
                    std::memcpy(&half[i], &hv, 2);
                }
            }
            ok = std::fwrite(half.data(), 2, o.n, f) == o.n;
        }
    }
    ok = (std::fclose(f) == 0) && ok;
    if (!ok || std::rename(tmp.c_str(), path) != 0) {
        std::remove(tmp.c_str());
        set_error(std::string("cannot write ") + path);
        return ERR_ARGUMENT;
    }
    return OK;
}

// Loads a checkpoint written by laya_trainer_save_checkpoint or by the reference's Save: every parameter must be
// present with its shape (F32, F16 or BF16); AdamW's state and step count are restored when the file has them and
// reset otherwise.  The bf16 copies the products read are rebuilt from the loaded masters.
int laya_trainer_restore_checkpoint(laya_trainer* t, const char* path) {
    if (!t || !path) { set_error("null argument"); return ERR_ARGUMENT; }
    std::FILE* f = std::fopen(path, "rb");
    if (!f) { set_error(std::string("cannot open ") + path); return ERR_NOT_FOUND; }
    st::Header h;
    std::string err;
    if (!st::read_header(f, &h, &err)) { std::fclose(f); set_error(std::string(path) + ": " + err); return ERR_ARGUMENT; }
    auto load = [&](const st::Entry& e, float* dst, size_t n, const std::string& name) -> int {
        const int es = st::elem_size(e.dtype);
        if (es == 0) { set_error(name + ": unsupported dtype " + e.dtype); return ERR_ARGUMENT; }
        int64_t count = 1;
        for (int64_t d : e.shape) count *= d;
        if (static_cast<size_t>(count) != n || e.end - e.begin != n * static_cast<uint64_t>(es)) {
            set_error(name + ": shape or size does not match the model");
            return ERR_ARGUMENT;
        }
        std::vector<unsigned char> raw(e.end - e.begin);
        if (std::fseek(f, static_cast<long>(h.data_start + e.begin), SEEK_SET) != 0 ||
            std::fread(raw.data(), 1, raw.size(), f) != raw.size()) {
            set_error(name + ": file shorter than its header says");
            return ERR_ARGUMENT;
        }
        if (es == 4) std::memcpy(dst, raw.data(), raw.size());
        else
            for (size_t i = 0; i < n; ++i) {
                uint16_t b;
                std::memcpy(&b, raw.data() + 2 * i, 2);
                if (e.dtype == "BF16") dst[i] = st::from_bf16(b);
                else { __half hv; std::memcpy(&hv, &b, 2); dst[i] = __half2float(hv); }
            }
        return OK;
    };
    std::vector<float> master(t->P, 0.f), m, v;
    bool have_opt = h.metadata.count("optimizer_step") > 0;
    if (have_opt) { m.assign(t->P, 0.f); v.assign(t->P, 0.f); }
    int rc = OK;
    for (Param& p : t->params) {
        const size_t n = static_cast<size_t>(p.rows * p.cols);
        auto it = h.tensors.find(p.name);
        if (it == h.tensors.end()) { set_error(std::string(path) + " has no tensor " + p.name); rc = ERR_NOT_FOUND; break; }
        if ((rc = load(it->second, master.data() + p.off, n, p.name)) != OK) break;
        p.stored = it->second.dtype == "BF16" ? LAYA_BF16 : it->second.dtype == "F16" ? LAYA_F16 : LAYA_F32;
        p.shape = it->second.shape;
        if (have_opt) {
            auto im = h.tensors.find("optimizer.m." + p.name), iv = h.tensors.find("optimizer.v." + p.name);
            if (im == h.tensors.end() || iv == h.tensors.end()) { set_error(std::string(path) + " lacks the optimizer state of " + p.name); rc = ERR_NOT_FOUND; break; }
            if ((rc = load(im->second, m.data() + p.off, n, im->first)) != OK) break;
            if ((rc = load(iv->second, v.data() + p.off, n, iv->first)) != OK) break;
        }
    }
    std::fclose(f);
    if (rc != OK) return rc;
    DeviceGuard g(t->device);
    if (t->comm.stream) LAYA_CUDA(cudaStreamSynchronize(t->comm.stream));
    LAYA_CUDA(cudaMemcpyAsync(t->master, master.data(), sizeof(float) * t->P, cudaMemcpyHostToDevice, t->stream));
    RC(f32_split_bf16(t->master, t->shadow, t->shadow_lo, t->P, t->stream));
    if (have_opt) {
        LAYA_CUDA(cudaMemcpyAsync(t->m, m.data(), sizeof(float) * t->P, cudaMemcpyHostToDevice, t->stream));
        LAYA_CUDA(cudaMemcpyAsync(t->v, v.data(), sizeof(float) * t->P, cudaMemcpyHostToDevice, t->stream));
        t->steps = std::strtoll(h.metadata["optimizer_step"].c_str(), nullptr, 10);
    } else {
        LAYA_CUDA(cudaMemsetAsync(t->m, 0, sizeof(float) * t->P, t->stream));
        LAYA_CUDA(cudaMemsetAsync(t->v, 0, sizeof(float) * t->P, t->stream));
        t->steps = 0;
    }
    LAYA_CUDA(cudaStreamSynchronize(t->stream));
    return OK;
}

int laya_trainer_param_count(laya_trainer* t, int64_t* total, int64_t* trainable) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    int64_t a = 0, b = 0;
    for (const auto& p : t->params) {
        a += p.rows * p.cols;
        if (p.trainable) b += p.rows * p.cols;
    }
    if (total) *total = a;
    if (trainable) *trainable = b;
    return OK;
}

int laya_trainer_param_info(laya_trainer* t, int index, const char** name, int64_t* rows, int64_t* cols) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    if (index < 0 || index >= static_cast<int>(t->params.size())) {
        set_error("parameter index out of range");
        return ERR_OUT_OF_RANGE;
    }
    const Param& p = t->params[index];
    if (name) *name = p.name.c_str();
    if (rows) *rows = p.rows;
    if (cols) *cols = p.cols;
    return OK;
}

// ------------------------------------------------------------------------------------------------ batches
int laya_batch_create(laya_trainer* t, laya_batch** out) {
    if (!t || !out) { set_error("null argument"); return ERR_ARGUMENT; }
    *out = nullptr;
    DeviceGuard g(t->device);
    static std::atomic<uint64_t> next_id{0};
    laya_batch* b = new laya_batch();
    b->owner = t;
    b->device = t->device;
    b->id = ++next_id;
    size_t o = 0;
    auto take = [&](size_t bytes) { const size_t r = o; o += (bytes + 255) & ~size_t(255); return r; };
    const size_t T = t->Tc, N = t->Nc, M = t->Mc, TL = t->tiles_cap;
    b->o_ids = take(4 * T); b->o_seg_start = take(4 * N); b->o_seg_len = take(4 * N); b->o_qtype = take(4 * N);
    b->o_tok_item = take(4 * T); b->o_tile_item = take(4 * TL); b->o_tile_p0 = take(4 * TL); b->o_n_tiles = take(4);
    b->o_marker_rows = take(4 * M); b->o_mk_start = take(4 * N); b->o_mk_count = take(4 * N);
    b->o_tq_item = take(4 * TL); b->o_tq_p0 = take(4 * TL); b->o_n_tq = take(4);
    b->o_tp_item = take(4 * TL); b->o_tp_p0 = take(4 * TL); b->o_n_tp = take(4);
    b->o_targets = take(4 * M); b->o_draws = take(8 * MAX_GROUPS * M);
    b->bytes = o;
    if (cudaMalloc(&b->dev, o) != cudaSuccess || cudaMallocHost(&b->host, o) != cudaSuccess ||
        cudaEventCreateWithFlags(&b->staged, cudaEventDisableTiming) != cudaSuccess) {
        const int rc = cuda_fail(cudaGetLastError(), "batch allocation");
        laya_batch_destroy(b);
        return rc;
    }
    char* base = static_cast<char*>(b->dev);
    b->ids = reinterpret_cast<int32_t*>(base + b->o_ids);
    b->seg_start = reinterpret_cast<int32_t*>(base + b->o_seg_start);
    b->seg_len = reinterpret_cast<int32_t*>(base + b->o_seg_len);
    b->qtype = reinterpret_cast<int32_t*>(base + b->o_qtype);
    b->tok_item = reinterpret_cast<int32_t*>(base + b->o_tok_item);
    b->tile_item = reinterpret_cast<int32_t*>(base + b->o_tile_item);
    b->tile_p0 = reinterpret_cast<int32_t*>(base + b->o_tile_p0);
    b->n_tiles = reinterpret_cast<int32_t*>(base + b->o_n_tiles);
    b->marker_rows = reinterpret_cast<int32_t*>(base + b->o_marker_rows);
    b->mk_start = reinterpret_cast<int32_t*>(base + b->o_mk_start);
    b->mk_count = reinterpret_cast<int32_t*>(base + b->o_mk_count);
    b->tq_item = reinterpret_cast<int32_t*>(base + b->o_tq_item);
    b->tq_p0 = reinterpret_cast<int32_t*>(base + b->o_tq_p0);
    b->n_tq = reinterpret_cast<int32_t*>(base + b->o_n_tq);
    b->tp_item = reinterpret_cast<int32_t*>(base + b->o_tp_item);
    b->tp_p0 = reinterpret_cast<int32_t*>(base + b->o_tp_p0);
    b->n_tp = reinterpret_cast<int32_t*>(base + b->o_n_tp);
    b->targets = reinterpret_cast<float*>(base + b->o_targets);
    b->draws = reinterpret_cast<double*>(base + b->o_draws);
    *out = b;
    return OK;
}

int laya_batch_destroy(laya_batch* b) {
    if (!b) return OK;
    DeviceGuard g(b->device);
    if (b->staged) { cudaEventSynchronize(b->staged); cudaEventDestroy(b->staged); }
    if (b->dev) cudaFree(b->dev);
    if (b->host) cudaFreeHost(b->host);
    delete b;
    return OK;
}

int laya_batch_set(laya_trainer* t, laya_batch* b, const int32_t* ids, const int32_t* seg_len, const int32_t* qtype,
                   int n_items, const int32_t* marker_count, const int32_t* markers, const float* targets,
                   const double* draws, int groups) {
    if (!t || !b || b->owner != t) { set_error("batch does not belong to this trainer"); return ERR_ARGUMENT; }
    if (!ids || !seg_len || !qtype || !marker_count || !markers) { set_error("null argument"); return ERR_ARGUMENT; }
    if (n_items <= 0 || n_items > t->Nc) { set_error("item count outside [1, max_items]"); return ERR_ARGUMENT; }
    if (groups < 0 || groups > MAX_GROUPS || (groups > 0 && !draws)) { set_error("noise groups outside [0, 16]"); return ERR_ARGUMENT; }
    int64_t T = 0, M = 0;
    for (int i = 0; i < n_items; ++i) {
        if (seg_len[i] <= 0 || seg_len[i] > t->maxpos) { set_error("segment length outside [1, max_segment]"); return ERR_ARGUMENT; }
        if (marker_count[i] <= 0) { set_error("every item needs at least one option marker"); return ERR_ARGUMENT; }
        if (qtype[i] < 0 || qtype[i] > 2) { set_error("question type outside [0, 3)"); return ERR_OUT_OF_RANGE; }
        T += seg_len[i];
        M += marker_count[i];
    }
    if (T > t->Tc) { set_error("batch exceeds max_tokens"); return ERR_ARGUMENT; }
    if (M > t->Mc) { set_error("batch exceeds max_markers"); return ERR_ARGUMENT; }
    for (int64_t i = 0; i < T; ++i)
        if (ids[i] < 0 || ids[i] >= t->V) {
            set_error("token id " + std::to_string(ids[i]) + " is outside the vocabulary.");
            return ERR_OUT_OF_RANGE;
        }
    DeviceGuard g(t->device);
    LAYA_CUDA(cudaEventSynchronize(b->staged));   // the previous copy out of the staging buffer is done
    char* h = static_cast<char*>(b->host);
    int32_t* hs = reinterpret_cast<int32_t*>(h + b->o_seg_start);
    int32_t* hl = reinterpret_cast<int32_t*>(h + b->o_seg_len);
    int32_t* hq = reinterpret_cast<int32_t*>(h + b->o_qtype);
    int32_t* hti = reinterpret_cast<int32_t*>(h + b->o_tok_item);
    int32_t* hit = reinterpret_cast<int32_t*>(h + b->o_tile_item);
    int32_t* hp0 = reinterpret_cast<int32_t*>(h + b->o_tile_p0);
    int32_t* hmr = reinterpret_cast<int32_t*>(h + b->o_marker_rows);
    int32_t* hms = reinterpret_cast<int32_t*>(h + b->o_mk_start);
    int32_t* hmc = reinterpret_cast<int32_t*>(h + b->o_mk_count);
    int32_t* hqi = reinterpret_cast<int32_t*>(h + b->o_tq_item);
    int32_t* hqp = reinterpret_cast<int32_t*>(h + b->o_tq_p0);
    int32_t* hpi = reinterpret_cast<int32_t*>(h + b->o_tp_item);
    int32_t* hpp = reinterpret_cast<int32_t*>(h + b->o_tp_p0);
    std::memcpy(h + b->o_ids, ids, sizeof(int32_t) * T);
    int start = 0, mk = 0, tiles = 0, tq = 0;
    double pg = 0, pl = 0;
    for (int i = 0; i < n_items; ++i) {
        const double L = seg_len[i];
        pg += L * L;
        for (int q = 0; q < seg_len[i]; ++q)
            pl += std::min(seg_len[i], q + t->window + 1) - std::max(0, q - t->window);
    }
    for (int i = 0; i < n_items; ++i) {
        hs[i] = start; hl[i] = seg_len[i]; hq[i] = qtype[i]; hms[i] = mk; hmc[i] = marker_count[i];
        for (int p = 0; p < seg_len[i]; ++p) hti[start + p] = i;
        for (int p0 = 0; p0 < seg_len[i]; p0 += 64) { hit[tiles] = i; hp0[tiles] = p0; ++tiles; }
        for (int p0 = 0; p0 < seg_len[i]; p0 += 128) { hqi[tq] = i; hqp[tq] = p0; ++tq; }
        for (int k = 0; k < marker_count[i]; ++k) {
            const int pos = std::max(0, markers[mk + k]);   // TrainableDecisionModel.cs:275
            if (pos >= seg_len[i]) { set_error("marker position past the end of its segment"); return ERR_OUT_OF_RANGE; }
            hmr[mk + k] = start + pos;
        }
        start += seg_len[i];
        mk += marker_count[i];
    }
    *reinterpret_cast<int32_t*>(h + b->o_n_tiles) = tiles;
    *reinterpret_cast<int32_t*>(h + b->o_n_tq) = tq;
    // pair tiles, longest segments first (a persistent CTA walks them in this order: the long items start first)
    std::vector<int> order(n_items);
    for (int i = 0; i < n_items; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) { return seg_len[x] > seg_len[y]; });
    int tp = 0;
    for (int i : order)
        for (int p0 = 0; p0 < seg_len[i]; p0 += 256) { hpi[tp] = i; hpp[tp] = p0; ++tp; }
    *reinterpret_cast<int32_t*>(h + b->o_n_tp) = tp;
    if (targets) std::memcpy(h + b->o_targets, targets, sizeof(float) * M);
    else std::memset(h + b->o_targets, 0, sizeof(float) * M);
    if (groups > 0) {
        double* hd = reinterpret_cast<double*>(h + b->o_draws);
        for (int gi = 0; gi < groups; ++gi) std::memcpy(hd + static_cast<size_t>(gi) * M, draws + static_cast<size_t>(gi) * M,
                                                        sizeof(double) * M);
    }
    b->T = static_cast<int>(T); b->n = n_items; b->M = static_cast<int>(M); b->tiles = tiles; b->groups = groups;
    b->tq = tq;
    b->tp = tp;
    b->pairs_global = pg;
    b->pairs_local = pl;
    b->version++;
    // one copy of the used prefix of the layout (draws last: copy exactly what this batch uses)
    const size_t used = b->o_draws + sizeof(double) * static_cast<size_t>(groups) * M;
    LAYA_CUDA(cudaMemcpyAsync(b->dev, b->host, used, cudaMemcpyHostToDevice, t->stream));
    LAYA_CUDA(cudaEventRecord(b->staged, t->stream));
    return OK;
}

int laya_batch_shape(laya_batch* b, int* tokens, int* items, int* options) {
    if (!b) { set_error("null batch"); return ERR_ARGUMENT; }
    if (tokens) *tokens = b->T;
    if (items) *items = b->n;
    if (options) *options = b->M;
    return OK;
}

// ------------------------------------------------------------------------------------------------ the step
int laya_train_forward(laya_trainer* t, laya_batch* b, int training, uint64_t seed, float* logits) {
    if (!t || !b || b->owner != t) { set_error("batch does not belong to this trainer"); return ERR_ARGUMENT; }
    if (b->T <= 0) { set_error("empty batch"); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    t->fwd_id = b->id;
    t->fwd_version = b->version;
    t->fwd_training = training != 0;
    t->fwd_seed = seed;
    t->have_logits = false;
    t->have_dlogits = false;
    RC(forward(t, b));
    t->have_logits = true;
    if (logits) {
        LAYA_CUDA(cudaMemcpyAsync(logits, t->logits, sizeof(float) * b->M, cudaMemcpyDeviceToHost, t->stream));
        RC(check_device_error(t));
    }
    return OK;
}

int laya_train_objective(laya_trainer* t, laya_batch* b, const laya_rlcd_desc* o, double* result, float* dlogits) {
    if (!t || !b || !o) { set_error("null argument"); return ERR_ARGUMENT; }
    if (!t->have_logits || t->fwd_id != b->id || t->fwd_version != b->version) {
        set_error("objective needs a forward of this batch first");
        return ERR_ARGUMENT;
    }
    if (o->groups <= 0 || o->groups != b->groups) { set_error("noise groups differ from the batch's draws"); return ERR_ARGUMENT; }
    if (!(o->sigma > 0)) { set_error("sigma must be positive"); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    tr::RlcdArgs a{};
    a.n_items = b->n; a.groups = o->groups; a.M = b->M;
    a.mk_start = b->mk_start; a.mk_count = b->mk_count; a.qtype = b->qtype;
    a.logits = t->logits; a.targets = b->targets; a.draws = b->draws;
    a.sigma = o->sigma; a.scale = o->scale; a.w_sph = o->spherical_weight; a.w_rps = o->rps_weight;
    a.w_ce = o->cross_entropy_weight;
    a.scratch = t->rl_scratch; a.dlogits = t->dlog; a.result = t->red + 4;
    RC(rlcd(a, t->stream));
    t->have_dlogits = true;
    if (dlogits) LAYA_CUDA(cudaMemcpyAsync(dlogits, t->dlog, sizeof(float) * b->M, cudaMemcpyDeviceToHost, t->stream));
    if (result) LAYA_CUDA(cudaMemcpyAsync(t->h_red + 4, t->red + 4, sizeof(double) * 4, cudaMemcpyDeviceToHost, t->stream));
    if (result || dlogits) {
        LAYA_CUDA(cudaStreamSynchronize(t->stream));
        if (result) std::memcpy(result, t->h_red + 4, sizeof(double) * 4);
    }
    return OK;
}

int laya_train_backward(laya_trainer* t, laya_batch* b, const float* dlogits) {
    if (!t || !b) { set_error("null argument"); return ERR_ARGUMENT; }
    if (!t->have_logits || t->fwd_id != b->id || t->fwd_version != b->version) {
        set_error("backward needs a forward of this batch first");
        return ERR_ARGUMENT;
    }
    DeviceGuard g(t->device);
    if (dlogits) {
        LAYA_CUDA(cudaMemcpyAsync(t->dlog, dlogits, sizeof(float) * b->M, cudaMemcpyHostToDevice, t->stream));
        LAYA_CUDA(cudaStreamSynchronize(t->stream));   // the host array may be reused as soon as we return
    } else if (!t->have_dlogits) {
        set_error("no logit gradients: run laya_train_objective or pass dlogits");
        return ERR_ARGUMENT;
    }
    const int accum = t->td.grad_accumulation > 0 ? t->td.grad_accumulation : 1;
    Comm& c = t->comm;
    c.active = c.comm && ((t->micro + 1) % accum == 0) && !c.reduced;
    c.next = 0;
    const int rc = backward(t, b);
    if (c.active && rc == OK) c.reduced = true;
    c.active = false;
    t->micro++;
    return rc;
}

int laya_train_set_lr(laya_trainer* t, const double* lr, int ngroups) {
    if (!t || !lr || ngroups < 1 || ngroups > 2) { set_error("two learning rates expected (encoder, head)"); return ERR_ARGUMENT; }
    t->lr[0] = lr[0];
    t->lr[1] = ngroups > 1 ? lr[1] : lr[0];
    return OK;
}

int laya_train_clip_and_step(laya_trainer* t, double max_norm, double* norm) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    cudaStream_t s = t->stream;
    Comm& c = t->comm;
    if (c.comm) {
        if (!c.reduced) RC(reduce_all(t));
        LAYA_CUDA(cudaEventRecord(c.done, c.stream));
        LAYA_CUDA(cudaStreamWaitEvent(s, c.done, 0));
    }
    const size_t tb = t->enc_train_begin;
    const int world = c.comm ? c.world : 1;
    LAYA_CUDA(cudaMemsetAsync(t->red, 0, sizeof(double) * 3, s));
    if (max_norm > 0 || norm) {
        RC(sumsq(t->grad + tb, t->P - tb, t->red + 8, s));
        RC(clip_scale(t->red + 8, max_norm > 0 ? max_norm : 1e300, world, t->red, t->red + 1, t->red + 2, s));
    } else if (world > 1) {
        const double inv = 1.0 / world;
        LAYA_CUDA(cudaMemcpyAsync(t->red + 1, &inv, sizeof(double), cudaMemcpyHostToDevice, s));
        LAYA_CUDA(cudaStreamSynchronize(s));
    }
    const bool scaled = max_norm > 0 || norm || world > 1;
    // AdamW.Step (AdamW.cs:29-73): one contiguous range per group
    t->steps++;
    const double c1 = 1.0 - std::pow(t->td.beta1, static_cast<double>(t->steps));
    const double c2 = 1.0 - std::pow(t->td.beta2, static_cast<double>(t->steps));
    const size_t ranges[2][2] = {{tb, t->enc_end}, {t->head_begin, t->P}};
    for (int gi = 0; gi < 2; ++gi) {
        const size_t a0 = ranges[gi][0], a1 = ranges[gi][1];
        if (a1 <= a0) continue;
        tr::AdamArgs a{};
        a.n = a1 - a0;
        a.param = t->master + a0; a.grad = t->grad + a0; a.m = t->m + a0; a.v = t->v + a0; a.shadow = t->shadow + a0;
        a.shadow_lo = t->shadow_lo ? t->shadow_lo + a0 : nullptr;
        a.decay = static_cast<float>(1.0 - t->lr[gi] * t->td.weight_decay);
        a.b1 = static_cast<float>(t->td.beta1); a.b2 = static_cast<float>(t->td.beta2);
        a.step_size = static_cast<float>(t->lr[gi] / c1);
        a.sqrt_c2 = static_cast<float>(std::sqrt(c2));
        a.eps = static_cast<float>(t->td.eps);
        a.gscale = scaled ? t->red + 1 : nullptr;
        RC(adamw(a, s));
    }
    c.reduced = false;
    t->micro = 0;
    if (norm) {
        LAYA_CUDA(cudaMemcpyAsync(t->h_red + 2, t->red + 2, sizeof(double), cudaMemcpyDeviceToHost, s));
        RC(check_device_error(t));
        *norm = t->h_red[2];
    }
    return OK;
}

int laya_train_zero_grads(laya_trainer* t) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    LAYA_CUDA(cudaMemsetAsync(t->grad, 0, sizeof(float) * t->P, t->stream));
    return OK;
}

int laya_train_steps(laya_trainer* t, int64_t* steps) {
    if (!t || !steps) { set_error("null argument"); return ERR_ARGUMENT; }
    *steps = t->steps;
    return OK;
}

int laya_trainer_launches(laya_trainer* t, long long* count) {
    if (!t || !count) { set_error("null argument"); return ERR_ARGUMENT; }
    *count = launches();
    return OK;
}

int laya_trainer_set_profiling(laya_trainer* t, int enabled) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    RC(collect_profile(t));
    t->profiling = enabled != 0;
    for (int k = 0; k < 3; ++k) { t->prof_ms[k] = t->prof_flops[k] = 0; t->prof_n[k] = 0; }
    return OK;
}

int laya_trainer_profile(laya_trainer* t, int kind, double* ms, double* flops, long long* n) {
    if (!t) { set_error("null trainer"); return ERR_ARGUMENT; }
    if (kind < 0 || kind > 2) { set_error("profile kind is 0 (products), 1 (attention forward) or 2 (backward)"); return ERR_ARGUMENT; }
    DeviceGuard g(t->device);
    RC(collect_profile(t));
    if (ms) *ms = t->prof_ms[kind];
    if (flops) *flops = t->prof_flops[kind];
    if (n) *n = t->prof_n[kind];
    t->prof_ms[kind] = t->prof_flops[kind] = 0;
    t->prof_n[kind] = 0;
    return OK;
}

int laya_comm_unique_id(void* id128) {
    if (!id128) { set_error("null argument"); return ERR_ARGUMENT; }
    RC(load_nccl());
    ncclUniqueId id;
    ncclResult_t r = g_nccl.getUniqueId(&id);
    if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
    std::memcpy(id128, &id, sizeof(id));
    return OK;
}

int laya_train_comm_init(laya_trainer* t, const void* id128, int rank, int world) {
    if (!t || !id128) { set_error("null argument"); return ERR_ARGUMENT; }
    if (world < 1 || rank < 0 || rank >= world) { set_error("rank outside [0, world)"); return ERR_ARGUMENT; }
    if (t->comm.comm) { set_error("communicator already initialised"); return ERR_ARGUMENT; }
    if (world == 1) return OK;
    RC(load_nccl());
    DeviceGuard g(t->device);
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof(id));
    ncclResult_t r = g_nccl.commInitRank(&t->comm.comm, world, id, rank);
    if (r != ncclSuccess) { t->comm.comm = nullptr; return nccl_fail(r, "ncclCommInitRank"); }
    t->comm.rank = rank;
    t->comm.world = world;
    LAYA_CUDA(cudaStreamCreateWithFlags(&t->comm.stream, cudaStreamNonBlocking));
    LAYA_CUDA(cudaEventCreateWithFlags(&t->comm.ready, cudaEventDisableTiming));
    LAYA_CUDA(cudaEventCreateWithFlags(&t->comm.done, cudaEventDisableTiming));
    // buckets over the trainable range, from the top of the buffer (finished first) down
    t->comm.buckets.clear();
    for (size_t end = t->P; end > t->enc_train_begin;) {
        const size_t begin = end - std::min(end - t->enc_train_begin, BUCKET_ELEMS);
        t->comm.buckets.push_back({begin, end});
        end = begin;
    }
    return OK;
}

}  // extern "C"
