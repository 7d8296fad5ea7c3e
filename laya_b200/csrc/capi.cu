// capi.cu — the C ABI (include/laya_b200.h): contexts, weight upload, the Q8_0 entry points and the batched
// decision forward.  Host C++ only; every computation runs in the kernels of q8_gemm.cu, norm.cu,
// attention.cu and head.cu.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/laya_b200.h"
#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "train.h"

namespace laya {

// ------------------------------------------------------------------------------------------------ errors
static thread_local std::string g_error;
void set_error(const std::string& msg) { g_error = msg; }
const char* last_error() { return g_error.c_str(); }
int cuda_fail(cudaError_t e, const char* what) {
    set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return ERR_CUDA;
}

static thread_local long long g_launches = 0;
void count_launch(int n) { g_launches += n; }
long long launches() { return g_launches; }

// ------------------------------------------------------------------------------------------------ TMA maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols, bool swizzle128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) { set_error("cuTensorMapEncodeTiled unavailable"); return ERR_CUDA; }
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {row_stride_bytes};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    (void)elem_bytes;
    CUresult r = fn(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d) for a %llux%llu tile map", static_cast<int>(r),
                 static_cast<unsigned long long>(rows), static_cast<unsigned long long>(cols));
        set_error(buf);
        return ERR_CUDA;
    }
    return OK;
}

}  // namespace laya

using namespace laya;

// ------------------------------------------------------------------------------------------------ context

namespace {

struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
};

struct QWeight {
    q8::code_t* q = nullptr;   // [N, K] fp16-held codes
    float* d = nullptr;    // [K/32, ldw]
    int N = 0, K = 0, ldw = 0;
    bool geglu = false;    // rows stored in [32 input | 32 gate] groups
};

// A projection of the fp32-accurate path: the weight as hi = bf16(w) and lo = bf16(w − hi), lo dropped when every
// weight is a bf16 value (a bf16 checkpoint) — the product is then two passes instead of three.
struct BWeight {
    __nv_bfloat16* hi = nullptr;
    __nv_bfloat16* lo = nullptr;
    int N = 0, K = 0;
};

int round_up(int x, int m) { return (x + m - 1) / m * m; }

// GeGLU row order: group g of 64 rows = input rows [32g, 32g+32) then gate rows [I + 32g, I + 32g + 32).
int geglu_src_row(int p, int I) {
    const int g = p / 64, w = p % 64;
    return w < 32 ? g * 32 + w : I + g * 32 + (w - 32);
}

bool ends_with(const std::string& s, const char* suf) {
    const size_t n = strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

}  // namespace

struct laya_ctx {
    int device = 0;
    cudaStream_t own = nullptr, stream = nullptr;
    laya_model_desc d{};
    std::vector<int> kinds;    // 1 global, 0 sliding
    int* err = nullptr;

    std::map<std::string, DevBuf> f32;     // fp32 tensors by name (element count = bytes/4)
    std::map<std::string, QWeight> q8;     // Q8_0 projections by name
    std::map<std::string, BWeight> bw;     // fp32-accurate projections by name (LAYA_PRECISION_F32)

    // rotary tables [maxpos, 32]
    int maxpos = 0;
    float *cos_g = nullptr, *sin_g = nullptr, *cos_l = nullptr, *sin_l = nullptr;

    // workspace
    int T_cap = 0, ldx = 0, maxk = 0, max_qtiles = 0;
    float* h = nullptr;
    float* qkv = nullptr;
    q8::code_t *qa0 = nullptr, *qa1 = nullptr;
    float *da0 = nullptr, *da1 = nullptr;
    int32_t *ids = nullptr, *seg_len = nullptr, *qtype = nullptr, *mk_count = nullptr, *markers = nullptr;
    int32_t *seg_start = nullptr, *mk_start = nullptr, *qt_start = nullptr, *qt_item = nullptr, *qt_q0 = nullptr,
            *n_qt = nullptr, *tok_item = nullptr, *marker_row = nullptr, *marker_item = nullptr;
    float *logits = nullptr, *act = nullptr;
    // the tensor-core attention (head_dim 64): rotated fp16 q | k | v and the 128-row query tiles
    __half* qkv16 = nullptr;
    int max_tq = 0;
    int32_t *tq_start = nullptr, *tq_item = nullptr, *tq_p0 = nullptr, *n_tq = nullptr;
    // LAYA_PRECISION_F32 workspace: activations split into hi/lo bf16 parts, the widest projection output fp32
    __nv_bfloat16 *xh0 = nullptr, *xl0 = nullptr, *xh1 = nullptr, *xl1 = nullptr;
    float* wide = nullptr;

    // profiling of the Q8_0 products
    bool profiling = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> ev_pool;
    size_t ev_used = 0;
    std::vector<double> ev_ops;
    double prof_ms = 0, prof_ops = 0;
    long long prof_n = 0;

    // recorder
    bool record = false;
    std::map<std::string, DevBuf> rec;

    std::vector<void*> allocs;
    long long launches_base = 0;
};

namespace {

int dalloc(laya_ctx* c, void** p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
    c->allocs.push_back(*p);
    return OK;
}
template <class T>
int dalloc_t(laya_ctx* c, T** p, size_t count) {
    return dalloc(c, reinterpret_cast<void**>(p), count * sizeof(T));
}

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

const float* F(laya_ctx* c, const std::string& name) {
    auto it = c->f32.find(name);
    return it == c->f32.end() ? nullptr : static_cast<const float*>(it->second.p);
}

int need_f32(laya_ctx* c, const std::string& name, const float** out) {
    *out = F(c, name);
    if (!*out) { set_error("missing tensor " + name); return ERR_NOT_FOUND; }
    return OK;
}

// The projections the reference runs through PackedMatrix (ModernBertEncoder.Pack, DecisionModel.cs:61-72): Q8_0 in a
// Q8_0 context, split bf16 in an fp32 one.
bool is_projection(const std::string& n) {
    if (n.rfind("encoder.layers.", 0) == 0)
        return ends_with(n, "attn.Wqkv.weight") || ends_with(n, "attn.Wo.weight") || ends_with(n, "mlp.Wi.weight") ||
               ends_with(n, "mlp.Wo.weight");
    if (n.rfind("head.layers.", 0) == 0)
        return ends_with(n, "self_attn.in_proj_weight") || ends_with(n, "self_attn.out_proj.weight") ||
               ends_with(n, "linear1.weight") || ends_with(n, "linear2.weight");
    return false;
}
bool is_q8_projection(const laya_ctx* c, const std::string& n) {
    return c->d.precision == LAYA_PRECISION_Q8_0 && is_projection(n);
}

int check_device_error(laya_ctx* c) {
    int h = 0;
    LAYA_CUDA(cudaMemcpyAsync(&h, c->err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    if (h != 0) {
        LAYA_CUDA(cudaMemsetAsync(c->err, 0, sizeof(int), c->stream));
        LAYA_CUDA(cudaStreamSynchronize(c->stream));
        if (h == LAYA_DEV_ERR_TIMEOUT) { set_error("a device-side wait timed out"); return ERR_DEVICE_TIMEOUT; }
        set_error("index out of range (token id, segment length or marker position)");
        return ERR_OUT_OF_RANGE;
    }
    return OK;
}

int gemm_profiled(laya_ctx* c, const q8::GemmArgs& a) {
    if (!c->profiling) return q8::gemm(a, c->stream);
    if (c->ev_used == c->ev_pool.size()) {
        cudaEvent_t e0, e1;
        LAYA_CUDA(cudaEventCreate(&e0));
        LAYA_CUDA(cudaEventCreate(&e1));
        c->ev_pool.push_back({e0, e1});
    }
    auto& ev = c->ev_pool[c->ev_used++];
    LAYA_CUDA(cudaEventRecord(ev.first, c->stream));
    int rc = q8::gemm(a, c->stream);
    LAYA_CUDA(cudaEventRecord(ev.second, c->stream));
    c->ev_ops.push_back(2.0 * a.M * static_cast<double>(a.N) * a.K);
    return rc;
}

int collect_profile(laya_ctx* c) {
    if (c->ev_used == 0) return OK;
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    for (size_t i = 0; i < c->ev_used; ++i) {
        float ms = 0;
        LAYA_CUDA(cudaEventElapsedTime(&ms, c->ev_pool[i].first, c->ev_pool[i].second));
        c->prof_ms += ms;
        c->prof_ops += c->ev_ops[i];
        c->prof_n += 1;
    }
    c->ev_used = 0;
    c->ev_ops.clear();
    return OK;
}

// Projection y[M, N] = Q8(x) · W with a given epilogue.  x codes/scales live in (q, d) with stride ldx.
int q8_proj(laya_ctx* c, const std::string& name, const q8::code_t* qx, const float* dx, int M, const float* bias,
            int epi, float* out, int ldo, q8::code_t* qout, float* qsc) {
    auto it = c->q8.find(name);
    if (it == c->q8.end()) { set_error("missing Q8_0 projection " + name); return ERR_NOT_FOUND; }
    const QWeight& w = it->second;
    q8::GemmArgs a{};
    a.M = M; a.N = w.N; a.K = w.K;
    a.qx = qx; a.dx = dx; a.ldx = c->ldx;
    a.qw = w.q; a.dw = w.d; a.ldw = w.ldw;
    a.bias = bias; a.epi = epi;
    a.out = out; a.ldo = ldo;
    a.qout = qout; a.ldqo = (epi == q8::EPI_GEGLU_Q8) ? w.N / 2 : w.N;
    a.qsc = qsc; a.ldqs = c->ldx;
    a.err = c->err;
    return gemm_profiled(c, a);
}

// Projection of the fp32-accurate path: out[M, N] (fp32; epi EPI_F32 stores, EPI_F32_ADD adds into out) =
// (xh + xl) · (Wh + Wl)ᵀ + bias from the split operands (two or three bf16 passes, fp32 accumulation).
int bf_proj(laya_ctx* c, const std::string& name, const __nv_bfloat16* xh, const __nv_bfloat16* xl, int M,
            const float* bias, int epi, float* out, int ldo) {
    auto it = c->bw.find(name);
    if (it == c->bw.end()) { set_error("missing projection " + name); return ERR_NOT_FOUND; }
    const BWeight& w = it->second;
    bf::Args a{};
    a.M = M; a.N = w.N; a.K = w.K;
    a.A = xh; a.lda = w.K; a.a_mn = 0;
    a.B = w.hi; a.ldb = w.K; a.b_mn = 0;
    a.A2 = xl; a.B2 = w.lo;
    a.bias = bias; a.epi = epi; a.out = out; a.ldo = ldo; a.err = c->err;
    if (!c->profiling) return bf::gemm(a, c->stream);
    if (c->ev_used == c->ev_pool.size()) {
        cudaEvent_t e0, e1;
        LAYA_CUDA(cudaEventCreate(&e0));
        LAYA_CUDA(cudaEventCreate(&e1));
        c->ev_pool.push_back({e0, e1});
    }
    auto& ev = c->ev_pool[c->ev_used++];
    LAYA_CUDA(cudaEventRecord(ev.first, c->stream));
    const int rc = bf::gemm(a, c->stream);
    LAYA_CUDA(cudaEventRecord(ev.second, c->stream));
    c->ev_ops.push_back(2.0 * M * static_cast<double>(w.N) * w.K);
    return rc;
}

int record_copy(laya_ctx* c, const std::string& name, const float* src, size_t count) {
    if (!c->record) return OK;
    DevBuf& b = c->rec[name];
    if (b.bytes < count * sizeof(float)) {
        if (b.p) cudaFree(b.p);
        LAYA_CUDA(cudaMalloc(&b.p, count * sizeof(float)));
        b.bytes = count * sizeof(float);
    }
    LAYA_CUDA(cudaMemcpyAsync(b.p, src, count * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    return OK;
}

#define RC(x)                     \
    do {                          \
        int rc_ = (x);            \
        if (rc_ != OK) return rc_; \
    } while (0)

// Attention of the decision forward, the context out as Q8_0 codes in (qa1, da1) — or, when at.hi is set (the
// fp32-accurate path), as bf16 hi/lo parts there: the tensor-core kernel for head_dim 64 (the q, k, v rows rotated
// into fp16 first), the mma.sync kernel otherwise.
int attend_q8(laya_ctx* c, attn::Args& at, int T) {
    const bool split_out = at.hi != nullptr;   // the fp32-accurate path: hi/lo context instead of Q8_0 codes
    if (c->qkv16 && at.hidden == 64 * at.heads) {
        RC(attn_prep16(at.qkv, at.ld, T, at.hidden, at.heads, c->tok_item, c->seg_start, at.cosv, at.sinv, c->qkv16,
                       at.ld, c->stream));
        InferAttn ia{};
        ia.qkv16 = c->qkv16; ia.ld = at.ld; ia.hidden = at.hidden; ia.heads = at.heads; ia.T = T;
        ia.seg_start = c->seg_start; ia.seg_len = c->seg_len;
        ia.tq_item = c->tq_item; ia.tq_p0 = c->tq_p0; ia.n_tq = c->n_tq; ia.max_tq = c->max_tq;
        ia.window = at.window; ia.scale = at.scale;
        if (split_out) { ia.hi = at.hi; ia.lo = at.lo; }
        else { ia.q = c->qa1; ia.d = c->da1; ia.ldd = c->ldx; }
        ia.err = c->err;
        const int rc = flash_forward_tc_q8(ia, c->stream);
        if (rc != ERR_NOT_SUPPORTED) return rc;
    }
    if (!split_out) { at.q = c->qa1; at.d = c->da1; at.ldd = c->ldx; }
    return attention(at, c->max_qtiles, c->stream);
}

// One encoder layer of the fp32-accurate path: the same steps as encoder_layer below with split bf16 products.
int encoder_layer_f32(laya_ctx* c, int i, int T) {
    const int H = c->d.hidden, I = c->d.intermediate;
    const std::string p = "encoder.layers." + std::to_string(i) + ".";
    LnArgs ln{};
    ln.rows = T; ln.n = H; ln.x = c->h; ln.eps = c->d.norm_eps; ln.err = c->err;
    ln.w = F(c, p + "attn_norm.weight"); ln.b = F(c, p + "attn_norm.bias");
    ln.apply_ln = ln.w != nullptr;
    ln.hi = c->xh0; ln.lo = c->xl0;
    RC(ln_q8(ln, c->stream));
    RC(bf_proj(c, p + "attn.Wqkv.weight", c->xh0, c->xl0, T, F(c, p + "attn.Wqkv.bias"), bf::EPI_F32, c->qkv, 3 * H));
    const bool global = c->kinds[i] != 0;
    attn::Args at{};
    at.qkv = c->qkv; at.ld = 3 * H; at.hidden = H; at.heads = c->d.heads;
    at.seg_start = c->seg_start; at.seg_len = c->seg_len;
    at.qtile_item = c->qt_item; at.qtile_q0 = c->qt_q0; at.n_qtiles = c->n_qt;
    at.window = global ? -1 : c->d.local_attention / 2;
    at.scale = 1.0f / std::sqrt(static_cast<float>(H / c->d.heads));
    at.cosv = global ? c->cos_g : c->cos_l; at.sinv = global ? c->sin_g : c->sin_l;
    at.hi = c->xh0; at.lo = c->xl0;
    RC(attend_q8(c, at, T));
    RC(bf_proj(c, p + "attn.Wo.weight", c->xh0, c->xl0, T, F(c, p + "attn.Wo.bias"), bf::EPI_F32_ADD, c->h, H));
    RC(need_f32(c, p + "mlp_norm.weight", &ln.w));
    ln.b = F(c, p + "mlp_norm.bias"); ln.apply_ln = 1;
    RC(ln_q8(ln, c->stream));
    RC(bf_proj(c, p + "mlp.Wi.weight", c->xh0, c->xl0, T, F(c, p + "mlp.Wi.bias"), bf::EPI_F32, c->wide, 2 * I));
    RC(geglu_fwd_f32(c->wide, T, I, c->xh1, c->xl1, c->stream));
    RC(bf_proj(c, p + "mlp.Wo.weight", c->xh1, c->xl1, T, F(c, p + "mlp.Wo.bias"), bf::EPI_F32_ADD, c->h, H));
    return record_copy(c, "encoder.layers." + std::to_string(i) + ".output", c->h, static_cast<size_t>(T) * H);
}

// One decision-head layer of the fp32-accurate path (head_layer below, split bf16 products, ReLU in fp32).
int head_layer_f32(laya_ctx* c, int i, int T) {
    const int H = c->d.hidden;
    const std::string p = "head.layers." + std::to_string(i) + ".";
    LnArgs ln{};
    ln.rows = T; ln.n = H; ln.x = c->h; ln.eps = 1e-5f; ln.err = c->err; ln.apply_ln = 1;
    RC(need_f32(c, p + "norm1.weight", &ln.w));
    ln.b = F(c, p + "norm1.bias");
    ln.hi = c->xh0; ln.lo = c->xl0;
    RC(ln_q8(ln, c->stream));
    RC(bf_proj(c, p + "self_attn.in_proj_weight", c->xh0, c->xl0, T, F(c, p + "self_attn.in_proj_bias"), bf::EPI_F32,
               c->qkv, 3 * H));
    attn::Args at{};
    at.qkv = c->qkv; at.ld = 3 * H; at.hidden = H; at.heads = std::max(1, H / 64);
    at.seg_start = c->seg_start; at.seg_len = c->seg_len;
    at.qtile_item = c->qt_item; at.qtile_q0 = c->qt_q0; at.n_qtiles = c->n_qt;
    at.window = -1; at.cosv = nullptr; at.sinv = nullptr;
    at.scale = 1.0f / std::sqrt(static_cast<float>(H / at.heads));
    at.hi = c->xh0; at.lo = c->xl0;
    RC(attend_q8(c, at, T));
    RC(bf_proj(c, p + "self_attn.out_proj.weight", c->xh0, c->xl0, T, F(c, p + "self_attn.out_proj.bias"),
               bf::EPI_F32_ADD, c->h, H));
    RC(need_f32(c, p + "norm2.weight", &ln.w));
    ln.b = F(c, p + "norm2.bias");
    RC(ln_q8(ln, c->stream));
    RC(bf_proj(c, p + "linear1.weight", c->xh0, c->xl0, T, F(c, p + "linear1.bias"), bf::EPI_F32, c->wide, 4 * H));
    RC(relu_mask_f32(c->wide, c->xh1, c->xl1, static_cast<size_t>(T) * 4 * H, tr::Mask{0.0f, 1.0f, 0}, c->stream));
    RC(bf_proj(c, p + "linear2.weight", c->xh1, c->xl1, T, F(c, p + "linear2.bias"), bf::EPI_F32_ADD, c->h, H));
    return record_copy(c, "head.layers." + std::to_string(i) + ".output", c->h, static_cast<size_t>(T) * H);
}

// One encoder layer on c->h (ModernBertEncoder.Forward loop body, ModernBertEncoder.cs:155-183).
int encoder_layer(laya_ctx* c, int i, int T) {
    if (c->d.precision == LAYA_PRECISION_F32) return encoder_layer_f32(c, i, T);
    const int H = c->d.hidden;
    const std::string p = "encoder.layers." + std::to_string(i) + ".";
    LnArgs ln{};
    ln.rows = T; ln.n = H; ln.x = c->h; ln.eps = c->d.norm_eps; ln.err = c->err;
    ln.w = F(c, p + "attn_norm.weight"); ln.b = F(c, p + "attn_norm.bias");
    ln.apply_ln = ln.w != nullptr;
    ln.q = c->qa0; ln.d = c->da0; ln.ldd = c->ldx;
    RC(ln_q8(ln, c->stream));
    RC(q8_proj(c, p + "attn.Wqkv.weight", c->qa0, c->da0, T, F(c, p + "attn.Wqkv.bias"), q8::EPI_STORE, c->qkv, 3 * H,
               nullptr, nullptr));
    const bool global = c->kinds[i] != 0;
    attn::Args at{};
    at.qkv = c->qkv; at.ld = 3 * H; at.hidden = H; at.heads = c->d.heads;
    at.seg_start = c->seg_start; at.seg_len = c->seg_len;
    at.qtile_item = c->qt_item; at.qtile_q0 = c->qt_q0; at.n_qtiles = c->n_qt;
    at.window = global ? -1 : c->d.local_attention / 2;
    at.scale = 1.0f / std::sqrt(static_cast<float>(H / c->d.heads));
    at.cosv = global ? c->cos_g : c->cos_l; at.sinv = global ? c->sin_g : c->sin_l;
    RC(attend_q8(c, at, T));
    RC(q8_proj(c, p + "attn.Wo.weight", c->qa1, c->da1, T, F(c, p + "attn.Wo.bias"), q8::EPI_RESID, c->h, H, nullptr,
               nullptr));
    const float* mw;
    RC(need_f32(c, p + "mlp_norm.weight", &mw));
    ln.w = mw; ln.b = F(c, p + "mlp_norm.bias"); ln.apply_ln = 1;
    RC(ln_q8(ln, c->stream));
    RC(q8_proj(c, p + "mlp.Wi.weight", c->qa0, c->da0, T, F(c, p + "mlp.Wi.bias"), q8::EPI_GEGLU_Q8, nullptr, 0,
               c->qa1, c->da1));
    RC(q8_proj(c, p + "mlp.Wo.weight", c->qa1, c->da1, T, F(c, p + "mlp.Wo.bias"), q8::EPI_RESID, c->h, H, nullptr,
               nullptr));
    return record_copy(c, "encoder.layers." + std::to_string(i) + ".output", c->h, static_cast<size_t>(T) * H);
}

// One decision-head layer on c->h (DecisionModel.HeadForward, DecisionModel.cs:236-307).
int head_layer(laya_ctx* c, int i, int T) {
    if (c->d.precision == LAYA_PRECISION_F32) return head_layer_f32(c, i, T);
    const int H = c->d.hidden;
    const std::string p = "head.layers." + std::to_string(i) + ".";
    LnArgs ln{};
    ln.rows = T; ln.n = H; ln.x = c->h; ln.eps = 1e-5f; ln.err = c->err; ln.apply_ln = 1;
    RC(need_f32(c, p + "norm1.weight", &ln.w));
    ln.b = F(c, p + "norm1.bias");
    ln.q = c->qa0; ln.d = c->da0; ln.ldd = c->ldx;
    RC(ln_q8(ln, c->stream));
    RC(q8_proj(c, p + "self_attn.in_proj_weight", c->qa0, c->da0, T, F(c, p + "self_attn.in_proj_bias"),
               q8::EPI_STORE, c->qkv, 3 * H, nullptr, nullptr));
    attn::Args at{};
    at.qkv = c->qkv; at.ld = 3 * H; at.hidden = H; at.heads = std::max(1, H / 64);
    at.seg_start = c->seg_start; at.seg_len = c->seg_len;
    at.qtile_item = c->qt_item; at.qtile_q0 = c->qt_q0; at.n_qtiles = c->n_qt;
    at.window = -1; at.cosv = nullptr; at.sinv = nullptr;
    at.scale = 1.0f / std::sqrt(static_cast<float>(H / at.heads));
    RC(attend_q8(c, at, T));
    RC(q8_proj(c, p + "self_attn.out_proj.weight", c->qa1, c->da1, T, F(c, p + "self_attn.out_proj.bias"),
               q8::EPI_RESID, c->h, H, nullptr, nullptr));
    RC(need_f32(c, p + "norm2.weight", &ln.w));
    ln.b = F(c, p + "norm2.bias");
    RC(ln_q8(ln, c->stream));
    RC(q8_proj(c, p + "linear1.weight", c->qa0, c->da0, T, F(c, p + "linear1.bias"), q8::EPI_RELU_Q8, nullptr, 0,
               c->qa1, c->da1));
    RC(q8_proj(c, p + "linear2.weight", c->qa1, c->da1, T, F(c, p + "linear2.bias"), q8::EPI_RESID, c->h, H, nullptr,
               nullptr));
    return record_copy(c, "head.layers." + std::to_string(i) + ".output", c->h, static_cast<size_t>(T) * H);
}

int run_plan(laya_ctx* c, int n_items, int T, int n_markers) {
    PlanArgs pa{};
    pa.n_items = n_items; pa.n_tokens = T; pa.n_markers = n_markers; pa.max_qtiles = c->max_qtiles;
    pa.seg_len = c->seg_len; pa.marker_count = c->mk_count; pa.markers = c->markers;
    pa.seg_start = c->seg_start; pa.mk_start = c->mk_start; pa.qt_start = c->qt_start;
    pa.qt_item = c->qt_item; pa.qt_q0 = c->qt_q0; pa.n_qtiles = c->n_qt;
    pa.tok_item = c->tok_item; pa.marker_row = c->marker_row; pa.marker_item = c->marker_item;
    pa.err = c->err;
    pa.max_tq = c->max_tq; pa.tq_start = c->tq_start; pa.tq_item = c->tq_item; pa.tq_p0 = c->tq_p0; pa.n_tq = c->n_tq;
    return plan(pa, c->stream);
}

int encoder_body(laya_ctx* c, int T) {
    const int H = c->d.hidden;
    LnArgs ln{};
    ln.rows = T; ln.n = H; ln.ids = c->ids; ln.vocab = c->d.vocab; ln.eps = c->d.norm_eps; ln.err = c->err;
    RC(need_f32(c, "encoder.embeddings.tok_embeddings.weight", &ln.table));
    RC(need_f32(c, "encoder.embeddings.norm.weight", &ln.w));
    ln.b = F(c, "encoder.embeddings.norm.bias");
    ln.apply_ln = 1; ln.out = c->h;
    RC(ln_embed(ln, c->stream));
    for (int i = 0; i < c->d.layers; ++i) RC(encoder_layer(c, i, T));
    return OK;
}


// Device-side forward on already-staged inputs (c->ids, c->seg_len, c->qtype, c->mk_count, c->markers).
// encoder_only: stop after the final LayerNorm (ModernBertEncoder.Forward's result) in c->h.
int forward_staged(laya_ctx* c, int n_items, int T, int n_markers, float* logits_out, float* act_out,
                   bool encoder_only) {
    const int H = c->d.hidden;
    RC(run_plan(c, n_items, T, n_markers));
    RC(encoder_body(c, T));
    LnArgs ln{};
    ln.rows = T; ln.n = H; ln.x = c->h; ln.out = c->h; ln.eps = c->d.norm_eps; ln.err = c->err; ln.apply_ln = 1;
    RC(need_f32(c, "encoder.final_norm.weight", &ln.w));
    ln.b = F(c, "encoder.final_norm.bias");
    if (encoder_only) return ln_final(ln, c->stream);
    RC(need_f32(c, "type_emb.weight", &ln.temb));
    ln.tok_item = c->tok_item; ln.qtype = c->qtype;
    RC(ln_final(ln, c->stream));
    RC(record_copy(c, "head.input", c->h, static_cast<size_t>(T) * H));
    for (int i = 0; i < c->d.head_layers; ++i) RC(head_layer(c, i, T));

    ScorerArgs sa{};
    sa.n_markers = n_markers; sa.hidden = H; sa.h = c->h; sa.marker_row = c->marker_row;
    RC(need_f32(c, "scorer.0.weight", &sa.ln_w));
    RC(need_f32(c, "scorer.0.bias", &sa.ln_b));
    RC(need_f32(c, "scorer.1.weight", &sa.w1));
    RC(need_f32(c, "scorer.1.bias", &sa.b1));
    RC(need_f32(c, "scorer.3.weight", &sa.w2));
    RC(need_f32(c, "scorer.3.bias", &sa.b2));
    sa.logits = logits_out;
    sa.hid = c->qkv;   // [n_markers, hidden] scratch: the QKV buffer is free after the head layers
    RC(scorer(sa, c->stream));
    if (act_out) {
        ActArgs aa{};
        aa.n_items = n_items; aa.hidden = H; aa.act_hidden = c->d.act_hidden; aa.n_act = c->d.n_act;
        aa.max_k = c->d.max_markers;
        aa.h = c->h; aa.seg_start = c->seg_start; aa.mk_start = c->mk_start; aa.marker_count = c->mk_count;
        aa.logits = logits_out;
        RC(need_f32(c, "act_head.0.weight", &aa.w1));
        RC(need_f32(c, "act_head.0.bias", &aa.b1));
        RC(need_f32(c, "act_head.2.weight", &aa.w2));
        RC(need_f32(c, "act_head.2.bias", &aa.b2));
        aa.probs = act_out;
        RC(act_head(aa, c->stream));
    }
    return OK;
}

int check_forward_args(laya_ctx* c, int n_items, long long T, long long n_markers) {
    if (c->d.precision != LAYA_PRECISION_Q8_0 && c->d.precision != LAYA_PRECISION_F32) {
        set_error("unknown precision");
        return ERR_NOT_SUPPORTED;
    }
    if (n_items < 0 || n_items > c->d.max_items) { set_error("item count outside [0, max_items]"); return ERR_ARGUMENT; }
    if (T < 0 || T > c->T_cap) { set_error("token count outside [0, max_tokens]"); return ERR_ARGUMENT; }
    if (n_markers < 0 || n_markers > c->d.max_markers) { set_error("marker count outside [0, max_markers]"); return ERR_ARGUMENT; }
    return OK;
}

int stage_inputs(laya_ctx* c, const int32_t* ids, const int32_t* seg_len, const int32_t* qtype, int n_items,
                 const int32_t* marker_count, const int32_t* markers, long long* T_out, long long* M_out) {
    long long T = 0, M = 0;
    for (int i = 0; i < n_items; ++i) {
        if (seg_len[i] < 0) { set_error("negative segment length"); return ERR_ARGUMENT; }
        T += seg_len[i];
        if (marker_count) {
            if (marker_count[i] < 0) { set_error("negative marker count"); return ERR_ARGUMENT; }
            M += marker_count[i];
        }
        if (qtype && (qtype[i] < 0 || qtype[i] > 2)) { set_error("question type outside 0..2"); return ERR_OUT_OF_RANGE; }
    }
    RC(check_forward_args(c, n_items, T, M));
    for (long long t = 0; t < T; ++t)
        if (ids[t] < 0 || ids[t] >= c->d.vocab) {
            set_error("token id " + std::to_string(ids[t]) + " is outside the vocabulary.");
            return ERR_OUT_OF_RANGE;
        }
    if (marker_count) {
        long long m = 0;
        for (int i = 0; i < n_items; ++i)
            for (int j = 0; j < marker_count[i]; ++j, ++m)
                if (std::max(0, markers[m]) >= seg_len[i]) { set_error("marker position past its question"); return ERR_OUT_OF_RANGE; }
    }
    LAYA_CUDA(cudaMemcpyAsync(c->ids, ids, sizeof(int32_t) * T, cudaMemcpyHostToDevice, c->stream));
    LAYA_CUDA(cudaMemcpyAsync(c->seg_len, seg_len, sizeof(int32_t) * n_items, cudaMemcpyHostToDevice, c->stream));
    if (qtype) LAYA_CUDA(cudaMemcpyAsync(c->qtype, qtype, sizeof(int32_t) * n_items, cudaMemcpyHostToDevice, c->stream));
    if (marker_count) {
        LAYA_CUDA(cudaMemcpyAsync(c->mk_count, marker_count, sizeof(int32_t) * n_items, cudaMemcpyHostToDevice, c->stream));
        LAYA_CUDA(cudaMemcpyAsync(c->markers, markers, sizeof(int32_t) * M, cudaMemcpyHostToDevice, c->stream));
    } else {
        LAYA_CUDA(cudaMemsetAsync(c->mk_count, 0, sizeof(int32_t) * std::max(1, n_items), c->stream));
    }
    *T_out = T;
    *M_out = M;
    return OK;
}

// fp16 bits -> float (host), for laya_upload_q8_0.
float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0) {
        if (man == 0) bits = sign;
        else {
            int e = -1;
            do { man <<= 1; ++e; } while (!(man & 0x400u));
            bits = sign | (static_cast<uint32_t>(127 - 15 - e) << 23) | ((man & 0x3FFu) << 13);
        }
    } else if (exp == 31) bits = sign | 0x7F800000u | (man << 13);
    else bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}
float bf16_bits_to_float(uint16_t b) {
    uint32_t bits = static_cast<uint32_t>(b) << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// A projection of the fp32-accurate path from fp32 values: hi = bf16(w) (round to nearest even), lo = bf16(w − hi),
// lo kept only when some weight is not a bf16 value.
int store_split(laya_ctx* c, const std::string& name, int N, int K, const float* w) {
    const size_t n = static_cast<size_t>(N) * K;
    std::vector<__nv_bfloat16> hi(n), lo(n);
    bool exact = true;
    for (size_t i = 0; i < n; ++i) {
        hi[i] = __float2bfloat16_rn(w[i]);
        const float r = w[i] - __bfloat162float(hi[i]);
        lo[i] = __float2bfloat16_rn(r);
        exact = exact && r == 0.0f;
    }
    BWeight& b = c->bw[name];
    if (b.hi) cudaFree(b.hi);
    if (b.lo) cudaFree(b.lo);
    b = BWeight{};
    b.N = N; b.K = K;
    LAYA_CUDA(cudaMalloc(&b.hi, n * sizeof(__nv_bfloat16)));
    LAYA_CUDA(cudaMemcpyAsync(b.hi, hi.data(), n * sizeof(__nv_bfloat16), cudaMemcpyHostToDevice, c->stream));
    if (!exact) {
        LAYA_CUDA(cudaMalloc(&b.lo, n * sizeof(__nv_bfloat16)));
        LAYA_CUDA(cudaMemcpyAsync(b.lo, lo.data(), n * sizeof(__nv_bfloat16), cudaMemcpyHostToDevice, c->stream));
    }
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    return OK;
}

int store_q8(laya_ctx* c, const std::string& name, const int8_t* q_host, const float* d_rows_host, int N, int K,
             bool device_quantize, const float* w_host) {
    QWeight w;
    w.N = N; w.K = K; w.ldw = round_up(N, 128);
    w.geglu = ends_with(name, "mlp.Wi.weight") && name.rfind("encoder.layers.", 0) == 0;
    if (w.geglu && (N % 64 != 0 || (N / 2) % 32 != 0)) { set_error("Wi needs 2·I rows with I a multiple of 32"); return ERR_ARGUMENT; }
    auto old = c->q8.find(name);
    if (old != c->q8.end()) { cudaFree(old->second.q); cudaFree(old->second.d); c->q8.erase(old); }
    LAYA_CUDA(cudaMalloc(&w.q, sizeof(q8::code_t) * static_cast<size_t>(N) * K));
    LAYA_CUDA(cudaMalloc(&w.d, sizeof(float) * static_cast<size_t>(K / 32) * w.ldw));
    LAYA_CUDA(cudaMemsetAsync(w.d, 0, sizeof(float) * static_cast<size_t>(K / 32) * w.ldw, c->stream));
    const int I = N / 2;
    if (device_quantize) {
        // permute rows on the host, quantize on the device (row permutation commutes with per-row quantization)
        std::vector<float> perm;
        const float* src = w_host;
        if (w.geglu) {
            perm.resize(static_cast<size_t>(N) * K);
            for (int p = 0; p < N; ++p)
                memcpy(&perm[static_cast<size_t>(p) * K], w_host + static_cast<size_t>(geglu_src_row(p, I)) * K, sizeof(float) * K);
            src = perm.data();
        }
        float* dtmp = nullptr;
        LAYA_CUDA(cudaMalloc(&dtmp, sizeof(float) * static_cast<size_t>(N) * K));
        LAYA_CUDA(cudaMemcpyAsync(dtmp, src, sizeof(float) * static_cast<size_t>(N) * K, cudaMemcpyHostToDevice, c->stream));
        int rc = q8::quantize_weights(dtmp, N, K, w.q, w.d, w.ldw, c->stream);
        LAYA_CUDA(cudaStreamSynchronize(c->stream));
        cudaFree(dtmp);
        if (rc) return rc;
    } else {
        std::vector<int8_t> qp(static_cast<size_t>(N) * K);
        std::vector<float> dt(static_cast<size_t>(K / 32) * w.ldw, 0.0f);
        for (int p = 0; p < N; ++p) {
            const int r = w.geglu ? geglu_src_row(p, I) : p;
            memcpy(&qp[static_cast<size_t>(p) * K], q_host + static_cast<size_t>(r) * K, K);
            for (int b = 0; b < K / 32; ++b) dt[static_cast<size_t>(b) * w.ldw + p] = d_rows_host[static_cast<size_t>(r) * (K / 32) + b];
        }
        int8_t* q8tmp = nullptr;
        LAYA_CUDA(cudaMalloc(&q8tmp, qp.size()));
        LAYA_CUDA(cudaMemcpyAsync(q8tmp, qp.data(), qp.size(), cudaMemcpyHostToDevice, c->stream));
        int rc = q8::widen_codes(q8tmp, w.q, qp.size(), c->stream);
        LAYA_CUDA(cudaMemcpyAsync(w.d, dt.data(), sizeof(float) * dt.size(), cudaMemcpyHostToDevice, c->stream));
        LAYA_CUDA(cudaStreamSynchronize(c->stream));
        cudaFree(q8tmp);
        if (rc) return rc;
    }
    c->q8[name] = w;
    return OK;
}

}  // namespace

// ================================================================================================ C ABI
extern "C" {

const char* laya_last_error(void) { return last_error(); }
const char* laya_version(void) { return "laya_b200 0.1 (sm_100a)"; }

int laya_ctx_create(const laya_model_desc* desc, int device, laya_ctx** out) {
    if (!desc || !out) { set_error("null argument"); return ERR_ARGUMENT; }
    *out = nullptr;
    const laya_model_desc& d = *desc;
    if (d.hidden <= 0 || d.heads <= 0 || d.hidden % d.heads || (d.hidden / d.heads != 64 && d.hidden / d.heads != 32) ||
        d.layers < 0 ||
        d.vocab <= 0 || d.intermediate <= 0 || d.intermediate % 32 || d.hidden % 32 || d.max_tokens <= 0 ||
        d.max_items <= 0 || d.max_markers < 0 || d.head_layers < 0) {
        set_error("invalid model geometry (head_dim must be 32 or 64, hidden and intermediate multiples of 32)");
        return ERR_ARGUMENT;
    }
    int ndev = 0;
    LAYA_CUDA(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) { set_error("no such CUDA device"); return ERR_ARGUMENT; }
    cudaDeviceProp prop;
    LAYA_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) {
        set_error("laya_b200 kernels are built for sm_100a (B200); this device is sm_" + std::to_string(prop.major) +
                  std::to_string(prop.minor));
        return ERR_NOT_SUPPORTED;
    }
    DeviceGuard g(device);
    laya_ctx* c = new laya_ctx();
    c->device = device;
    c->d = d;
    c->d.layer_kinds = nullptr;
    if (c->d.act_hidden <= 0) c->d.act_hidden = 256;
    if (c->d.n_act <= 0) c->d.n_act = 2;
    if (c->d.global_every <= 0) c->d.global_every = 3;
    c->kinds.resize(d.layers);
    for (int i = 0; i < d.layers; ++i)
        c->kinds[i] = d.layer_kinds ? (d.layer_kinds[i] != 0) : (i % c->d.global_every == 0);
    auto fail = [&](int rc) { laya_ctx_destroy(c); return rc; };
    if (cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking) != cudaSuccess) return fail(cuda_fail(cudaGetLastError(), "cudaStreamCreate"));
    c->stream = c->own;
    int rc;
    if ((rc = dalloc_t(c, &c->err, 1))) return fail(rc);
    cudaMemsetAsync(c->err, 0, sizeof(int), c->stream);

    const int H = d.hidden, I = d.intermediate;
    c->T_cap = d.max_tokens;
    c->ldx = round_up(d.max_tokens, 128);
    c->maxk = std::max({H, I, 4 * H});
    c->max_qtiles = d.max_tokens / 64 + d.max_items + 1;
    const size_t T = c->T_cap, L = c->ldx;
    if ((rc = dalloc_t(c, &c->h, T * H)) || (rc = dalloc_t(c, &c->qkv, T * 3 * H)) ||
        (rc = dalloc_t(c, &c->qa0, L * H)) || (rc = dalloc_t(c, &c->qa1, L * c->maxk)) ||
        (rc = dalloc_t(c, &c->da0, (H / 32) * L)) || (rc = dalloc_t(c, &c->da1, (c->maxk / 32) * L)) ||
        (rc = dalloc_t(c, &c->ids, T)) || (rc = dalloc_t(c, &c->seg_len, d.max_items)) ||
        (rc = dalloc_t(c, &c->qtype, d.max_items)) || (rc = dalloc_t(c, &c->mk_count, d.max_items)) ||
        (rc = dalloc_t(c, &c->markers, std::max(1, d.max_markers))) ||
        (rc = dalloc_t(c, &c->seg_start, d.max_items)) || (rc = dalloc_t(c, &c->mk_start, d.max_items)) ||
        (rc = dalloc_t(c, &c->qt_start, d.max_items)) || (rc = dalloc_t(c, &c->qt_item, c->max_qtiles)) ||
        (rc = dalloc_t(c, &c->qt_q0, c->max_qtiles)) || (rc = dalloc_t(c, &c->n_qt, 1)) ||
        (rc = dalloc_t(c, &c->tok_item, T)) || (rc = dalloc_t(c, &c->marker_row, std::max(1, d.max_markers))) ||
        (rc = dalloc_t(c, &c->marker_item, std::max(1, d.max_markers))) ||
        (rc = dalloc_t(c, &c->logits, std::max(1, d.max_markers))) ||
        (rc = dalloc_t(c, &c->act, static_cast<size_t>(d.max_items) * c->d.n_act)))
        return fail(rc);
    c->max_tq = d.max_tokens / 128 + d.max_items + 1;
    if ((rc = dalloc_t(c, &c->tq_start, d.max_items)) || (rc = dalloc_t(c, &c->tq_item, c->max_tq)) ||
        (rc = dalloc_t(c, &c->tq_p0, c->max_tq)) || (rc = dalloc_t(c, &c->n_tq, 1)))
        return fail(rc);
    if (d.hidden / d.heads == 64 && (rc = dalloc_t(c, &c->qkv16, T * 3 * H))) return fail(rc);
    if (d.precision == LAYA_PRECISION_F32) {
        const size_t widest = std::max(2 * static_cast<size_t>(I), 4 * static_cast<size_t>(H));
        if ((rc = dalloc_t(c, &c->xh0, T * H)) || (rc = dalloc_t(c, &c->xl0, T * H)) ||
            (rc = dalloc_t(c, &c->xh1, T * c->maxk)) || (rc = dalloc_t(c, &c->xl1, T * c->maxk)) ||
            (rc = dalloc_t(c, &c->wide, T * widest)))
            return fail(rc);
    } else if (d.precision != LAYA_PRECISION_Q8_0) {
        set_error("unknown precision");
        return fail(ERR_ARGUMENT);
    }
    // activation scales padding rows read by the products must be finite: zero both scale buffers once
    cudaMemsetAsync(c->da0, 0, sizeof(float) * (H / 32) * L, c->stream);
    cudaMemsetAsync(c->da1, 0, sizeof(float) * (c->maxk / 32) * L, c->stream);

    // Rotary tables (RopeCache, ModernBertEncoder.cs:357-379): angles in double, stored fp32, [pos, head_dim/2].
    c->maxpos = d.max_tokens;
    const int hd = d.hidden / d.heads, half = hd / 2;
    std::vector<float> cg(static_cast<size_t>(c->maxpos) * half), sg(cg.size()), cl(cg.size()), sl(cg.size());
    for (int i = 0; i < half; ++i) {
        const double ig = 1.0 / std::pow(d.theta_global, 2.0 * i / hd);
        const double il = 1.0 / std::pow(d.theta_local, 2.0 * i / hd);
        for (int p = 0; p < c->maxpos; ++p) {
            cg[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(p * ig));
            sg[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(p * ig));
            cl[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(p * il));
            sl[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(p * il));
        }
    }
    if ((rc = dalloc_t(c, &c->cos_g, cg.size())) || (rc = dalloc_t(c, &c->sin_g, cg.size())) ||
        (rc = dalloc_t(c, &c->cos_l, cg.size())) || (rc = dalloc_t(c, &c->sin_l, cg.size())))
        return fail(rc);
    cudaMemcpyAsync(c->cos_g, cg.data(), sizeof(float) * cg.size(), cudaMemcpyHostToDevice, c->stream);
    cudaMemcpyAsync(c->sin_g, sg.data(), sizeof(float) * cg.size(), cudaMemcpyHostToDevice, c->stream);
    cudaMemcpyAsync(c->cos_l, cl.data(), sizeof(float) * cg.size(), cudaMemcpyHostToDevice, c->stream);
    cudaMemcpyAsync(c->sin_l, sl.data(), sizeof(float) * cg.size(), cudaMemcpyHostToDevice, c->stream);
    if (cudaStreamSynchronize(c->stream) != cudaSuccess) return fail(cuda_fail(cudaGetLastError(), "context setup"));
    *out = c;
    return OK;
}

int laya_ctx_destroy(laya_ctx* c) {
    if (!c) return OK;
    DeviceGuard g(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    for (void* p : c->allocs) cudaFree(p);
    for (auto& kv : c->f32) cudaFree(kv.second.p);
    for (auto& kv : c->q8) { cudaFree(kv.second.q); cudaFree(kv.second.d); }
    for (auto& kv : c->bw) { cudaFree(kv.second.hi); if (kv.second.lo) cudaFree(kv.second.lo); }
    for (auto& kv : c->rec) cudaFree(kv.second.p);
    for (auto& e : c->ev_pool) { cudaEventDestroy(e.first); cudaEventDestroy(e.second); }
    if (c->own) cudaStreamDestroy(c->own);
    delete c;
    return OK;
}

int laya_ctx_set_stream(laya_ctx* c, void* stream) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    c->stream = static_cast<cudaStream_t>(stream);   // NULL: CUDA's legacy default stream
    return OK;
}

int laya_ctx_get_stream(laya_ctx* c, void** stream) {
    if (!c || !stream) { set_error("null argument"); return ERR_ARGUMENT; }
    *stream = static_cast<void*>(c->stream);
    return OK;
}

int laya_ctx_synchronize(laya_ctx* c) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    return check_device_error(c);
}

int laya_ctx_launches(laya_ctx* c, long long* count) {
    if (!c || !count) { set_error("null argument"); return ERR_ARGUMENT; }
    *count = launches();
    return OK;
}

int laya_ctx_set_profiling(laya_ctx* c, int enabled) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    RC(collect_profile(c));
    c->profiling = enabled != 0;
    c->prof_ms = c->prof_ops = 0;
    c->prof_n = 0;
    return OK;
}

int laya_ctx_profile(laya_ctx* c, double* ms, double* ops, long long* n) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    RC(collect_profile(c));
    if (ms) *ms = c->prof_ms;
    if (ops) *ops = c->prof_ops;
    if (n) *n = c->prof_n;
    c->prof_ms = c->prof_ops = 0;
    c->prof_n = 0;
    return OK;
}

int laya_upload_tensor(laya_ctx* c, const char* name, int dtype, const int64_t* shape, int rank, const void* host) {
    if (!c || !name || !host || (rank > 0 && !shape) || rank < 0 || rank > 8) { set_error("invalid argument"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    int64_t count = 1;
    for (int i = 0; i < rank; ++i) {
        if (shape[i] < 0) { set_error("negative dimension"); return ERR_ARGUMENT; }
        count *= shape[i];
    }
    std::vector<float> tmp;
    const float* src = nullptr;
    switch (dtype) {
        case LAYA_F32: src = static_cast<const float*>(host); break;
        case LAYA_BF16: {
            tmp.resize(count);
            const uint16_t* b = static_cast<const uint16_t*>(host);
            for (int64_t i = 0; i < count; ++i) tmp[i] = bf16_bits_to_float(b[i]);
            src = tmp.data();
            break;
        }
        case LAYA_F16: {
            tmp.resize(count);
            const uint16_t* b = static_cast<const uint16_t*>(host);
            for (int64_t i = 0; i < count; ++i) tmp[i] = half_bits_to_float(b[i]);
            src = tmp.data();
            break;
        }
        default: set_error("unsupported dtype for a float tensor"); return ERR_ARGUMENT;
    }
    const std::string n(name);
    if (is_q8_projection(c, n)) {
        if (rank != 2 || shape[1] % 32) { set_error(n + ": a Q8_0 projection needs [out, in] with in a multiple of 32"); return ERR_ARGUMENT; }
        return store_q8(c, n, nullptr, nullptr, static_cast<int>(shape[0]), static_cast<int>(shape[1]), true, src);
    }
    if (c->d.precision == LAYA_PRECISION_F32 && is_projection(n)) {
        if (rank != 2 || shape[1] % 8) { set_error(n + ": a projection needs [out, in] with in a multiple of 8"); return ERR_ARGUMENT; }
        return store_split(c, n, static_cast<int>(shape[0]), static_cast<int>(shape[1]), src);
    }
    std::vector<float> perm;
    if (ends_with(n, "mlp.Wi.bias") && c->d.precision == LAYA_PRECISION_Q8_0) {
        const int N = static_cast<int>(count);
        perm.resize(N);
        for (int p = 0; p < N; ++p) perm[p] = src[geglu_src_row(p, N / 2)];
        src = perm.data();
    }
    DevBuf& b = c->f32[n];
    if (b.bytes != static_cast<size_t>(count) * sizeof(float)) {
        if (b.p) cudaFree(b.p);
        b.p = nullptr;
        LAYA_CUDA(cudaMalloc(&b.p, std::max<size_t>(16, count * sizeof(float))));
        b.bytes = count * sizeof(float);
    }
    LAYA_CUDA(cudaMemcpyAsync(b.p, src, count * sizeof(float), cudaMemcpyHostToDevice, c->stream));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    return OK;
}

int laya_upload_q8_0(laya_ctx* c, const char* name, const int8_t* q, const uint16_t* d_fp16, int N, int K) {
    if (!c || !name || !q || !d_fp16 || N <= 0 || K <= 0 || K % 32) { set_error("invalid Q8_0 upload"); return ERR_ARGUMENT; }
    if (c->d.precision != LAYA_PRECISION_Q8_0) { set_error("not a Q8_0 context"); return ERR_NOT_SUPPORTED; }
    DeviceGuard g(c->device);
    std::vector<float> d(static_cast<size_t>(N) * (K / 32));
    for (size_t i = 0; i < d.size(); ++i) d[i] = half_bits_to_float(d_fp16[i]);
    return store_q8(c, name, q, d.data(), N, K, false, nullptr);
}

int laya_download_tensor(laya_ctx* c, const char* name, float* host, int64_t count) {
    if (!c || !name || !host) { set_error("invalid argument"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    const std::string n(name);
    auto it = c->f32.find(n);
    if (it != c->f32.end()) {
        const int64_t have = static_cast<int64_t>(it->second.bytes / sizeof(float));
        if (count < have) { set_error("host buffer too small"); return ERR_ARGUMENT; }
        std::vector<float> tmp(have);
        LAYA_CUDA(cudaMemcpy(tmp.data(), it->second.p, have * sizeof(float), cudaMemcpyDeviceToHost));
        if (ends_with(n, "mlp.Wi.bias") && c->d.precision == LAYA_PRECISION_Q8_0)
            for (int p = 0; p < have; ++p) host[geglu_src_row(p, static_cast<int>(have / 2))] = tmp[p];
        else memcpy(host, tmp.data(), have * sizeof(float));
        return OK;
    }
    auto bt = c->bw.find(n);
    if (bt != c->bw.end()) {
        const BWeight& w = bt->second;
        const size_t m = static_cast<size_t>(w.N) * w.K;
        if (count < static_cast<int64_t>(m)) { set_error("host buffer too small"); return ERR_ARGUMENT; }
        std::vector<__nv_bfloat16> hi(m), lo(m);
        LAYA_CUDA(cudaMemcpy(hi.data(), w.hi, m * sizeof(__nv_bfloat16), cudaMemcpyDeviceToHost));
        if (w.lo) LAYA_CUDA(cudaMemcpy(lo.data(), w.lo, m * sizeof(__nv_bfloat16), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < m; ++i) host[i] = __bfloat162float(hi[i]) + (w.lo ? __bfloat162float(lo[i]) : 0.0f);
        return OK;
    }
    auto jt = c->q8.find(n);
    if (jt == c->q8.end()) { set_error("no tensor named " + n); return ERR_NOT_FOUND; }
    const QWeight& w = jt->second;
    if (count < static_cast<int64_t>(w.N) * w.K) { set_error("host buffer too small"); return ERR_ARGUMENT; }
    std::vector<uint16_t> q(static_cast<size_t>(w.N) * w.K);
    std::vector<float> d(static_cast<size_t>(w.K / 32) * w.ldw);
    LAYA_CUDA(cudaMemcpy(q.data(), w.q, sizeof(uint16_t) * q.size(), cudaMemcpyDeviceToHost));
    LAYA_CUDA(cudaMemcpy(d.data(), w.d, sizeof(float) * d.size(), cudaMemcpyDeviceToHost));
    for (int p = 0; p < w.N; ++p) {
        const int r = w.geglu ? geglu_src_row(p, w.N / 2) : p;
        for (int k = 0; k < w.K; ++k)
            host[static_cast<size_t>(r) * w.K + k] = half_bits_to_float(q[static_cast<size_t>(p) * w.K + k]) * d[static_cast<size_t>(k / 32) * w.ldw + p];
    }
    return OK;
}

// ------------------------------------------------------------------------------------------------ Q8_0 entry points
int laya_q8_0_quantize_activations_device(laya_ctx* c, const float* x, int rows, int stride, int K, uint16_t* q,
                                          float* d, int ldd) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    if (rows < 0 || ldd < rows) { set_error("scale stride below the row count"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    return q8::quantize_activations(x, rows, stride, K, reinterpret_cast<q8::code_t*>(q), d, ldd, c->stream);
}

int laya_q8_0_quantize_weights_device(laya_ctx* c, const float* w, int N, int K, uint16_t* q, float* d, int ldd) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    if (N < 0 || ldd < N) { set_error("scale stride below the column count"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    return q8::quantize_weights(w, N, K, reinterpret_cast<q8::code_t*>(q), d, ldd, c->stream);
}

int laya_q8_0_gemm_device(laya_ctx* c, const uint16_t* qx, const float* dx, int ldx, int M, const uint16_t* qw,
                          const float* dw, int ldw, int N, int K, const float* bias, float* out, int ldo) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    if (M < 0 || N < 0 || ldo < N) { set_error("output stride below the column count"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    q8::GemmArgs a{};
    a.M = M; a.N = N; a.K = K; a.dx = dx; a.ldx = ldx; a.dw = dw; a.ldw = ldw;
    a.qx = reinterpret_cast<const q8::code_t*>(qx); a.qw = reinterpret_cast<const q8::code_t*>(qw);
    a.bias = bias; a.epi = q8::EPI_STORE; a.out = out; a.ldo = ldo; a.err = c->err;
    return gemm_profiled(c, a);
}

int laya_pack_q8_0(laya_ctx* c, const char* name, int dtype, const void* host, int N, int K) {
    if (!c || !name || !host || N <= 0 || K <= 0) { set_error("invalid argument"); return ERR_ARGUMENT; }
    if (K % 32) { set_error("Q8_0 needs a multiple of 32 inputs, got " + std::to_string(K) + "."); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    const size_t count = static_cast<size_t>(N) * K;
    std::vector<float> tmp;
    const float* src = nullptr;
    if (dtype == LAYA_F32) src = static_cast<const float*>(host);
    else if (dtype == LAYA_BF16 || dtype == LAYA_F16) {
        tmp.resize(count);
        const uint16_t* b = static_cast<const uint16_t*>(host);
        for (size_t i = 0; i < count; ++i) tmp[i] = dtype == LAYA_BF16 ? bf16_bits_to_float(b[i]) : half_bits_to_float(b[i]);
        src = tmp.data();
    } else { set_error("unsupported dtype for a Q8_0 weight"); return ERR_ARGUMENT; }
    return store_q8(c, name, nullptr, nullptr, N, K, true, src);
}

int laya_q8_0_gemm_fused_device(laya_ctx* c, int epilogue, const uint16_t* qx, const float* dx, int ldx, int M,
                                const uint16_t* qw, const float* dw, int ldw, int N, int K, const float* bias, float* out,
                                int ldo, uint16_t* qout, float* qscale, int ldqs) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    if (epilogue < 0 || epilogue > 4) { set_error("unknown epilogue"); return ERR_ARGUMENT; }
    if ((epilogue <= 1 && (!out || ldo < N)) || (epilogue >= 2 && (!qout || !qscale || ldqs < M))) {
        set_error("missing or short output"); return ERR_ARGUMENT;
    }
    DeviceGuard g(c->device);
    q8::GemmArgs a{};
    a.M = M; a.N = N; a.K = K; a.dx = dx; a.ldx = ldx; a.dw = dw; a.ldw = ldw;
    a.qx = reinterpret_cast<const q8::code_t*>(qx); a.qw = reinterpret_cast<const q8::code_t*>(qw);
    a.bias = bias; a.epi = epilogue; a.out = out; a.ldo = ldo; a.qout = reinterpret_cast<q8::code_t*>(qout);
    a.ldqo = (epilogue == q8::EPI_GEGLU_Q8 || epilogue == q8::EPI_SWIGLU_Q8) ? N / 2 : N;
    a.qsc = qscale; a.ldqs = ldqs; a.err = c->err;
    return gemm_profiled(c, a);
}

static int q8_linear_impl(laya_ctx* c, const char* weight, const float* x, int rows, int input_stride,
                          const float* bias, float* y, int output_stride, bool host) {
    if (!c || !weight || (rows > 0 && (!x || !y))) { set_error("invalid argument"); return ERR_ARGUMENT; }
    auto it = c->q8.find(weight);
    if (it == c->q8.end()) { set_error(std::string("no Q8_0 projection named ") + weight); return ERR_NOT_FOUND; }
    const QWeight& w = it->second;
    if (rows < 0 || input_stride < w.K || output_stride < w.N) { set_error("input is too small"); return ERR_ARGUMENT; }
    if (rows > c->T_cap) { set_error("more rows than the context's max_tokens"); return ERR_ARGUMENT; }
    if (rows == 0) return OK;
    DeviceGuard g(c->device);
    const float* dxin = x;
    float* dyout = y;
    const float* dbias = bias;
    float* tmp = nullptr;
    const size_t xin = (static_cast<size_t>(rows) - 1) * input_stride + w.K;
    const size_t yout = (static_cast<size_t>(rows) - 1) * output_stride + w.N;
    if (host) {
        // stage through the qkv workspace: [x | y | bias]
        const size_t need = xin + yout + w.N + 8;
        if (need > static_cast<size_t>(c->T_cap) * 3 * c->d.hidden) {
            LAYA_CUDA(cudaMalloc(&tmp, need * sizeof(float)));
        }
        float* base = tmp ? tmp : c->qkv;
        float* dx_ = base;
        float* dy_ = base + (xin + 3) / 4 * 4;           // 16-byte aligned
        float* db_ = dy_ + (yout + 3) / 4 * 4;
        LAYA_CUDA(cudaMemcpyAsync(dx_, x, xin * sizeof(float), cudaMemcpyHostToDevice, c->stream));
        if (bias) LAYA_CUDA(cudaMemcpyAsync(db_, bias, w.N * sizeof(float), cudaMemcpyHostToDevice, c->stream));
        if (output_stride != w.N) LAYA_CUDA(cudaMemcpyAsync(dy_, y, yout * sizeof(float), cudaMemcpyHostToDevice, c->stream));
        dxin = dx_; dyout = dy_; dbias = bias ? db_ : nullptr;
    }
    // activation codes [rows, K] and scales [K/32, ldx]: the workspace holds K <= maxk; wider inputs get their own
    q8::code_t* qa = c->qa1;
    float* da = c->da1;
    q8::code_t* qa_tmp = nullptr;
    float* da_tmp = nullptr;
    if (w.K > c->maxk) {
        LAYA_CUDA(cudaMalloc(&qa_tmp, sizeof(q8::code_t) * static_cast<size_t>(c->ldx) * w.K));
        LAYA_CUDA(cudaMalloc(&da_tmp, sizeof(float) * static_cast<size_t>(w.K / 32) * c->ldx));
        LAYA_CUDA(cudaMemsetAsync(da_tmp, 0, sizeof(float) * static_cast<size_t>(w.K / 32) * c->ldx, c->stream));
        qa = qa_tmp;
        da = da_tmp;
    }
    // The product stores whole 16-byte-aligned rows with the TMA; an output whose base or row stride does not allow
    // that (the reference accepts any stride) gets an aligned buffer and a strided copy.
    float* gout = dyout;
    int gld = output_stride;
    float* out_tmp = nullptr;
    if ((reinterpret_cast<uintptr_t>(dyout) & 15) || (output_stride & 3)) {
        gld = (w.N + 3) / 4 * 4;
        LAYA_CUDA(cudaMalloc(&out_tmp, sizeof(float) * static_cast<size_t>(rows) * gld));
        gout = out_tmp;
    }
    int rc = q8::quantize_activations(dxin, rows, input_stride, w.K, qa, da, c->ldx, c->stream);
    if (rc == OK) {
        q8::GemmArgs a{};
        a.M = rows; a.N = w.N; a.K = w.K; a.qx = qa; a.dx = da; a.ldx = c->ldx;
        a.qw = w.q; a.dw = w.d; a.ldw = w.ldw; a.bias = dbias; a.epi = q8::EPI_STORE; a.out = gout; a.ldo = gld;
        a.err = c->err;
        if (w.geglu) { set_error("Wi is stored in GeGLU row order; use the forward"); rc = ERR_NOT_SUPPORTED; }
        else rc = gemm_profiled(c, a);
    }
    if (rc == OK && out_tmp) {
        cudaError_t e = cudaMemcpy2DAsync(dyout, sizeof(float) * output_stride, out_tmp, sizeof(float) * gld,
                                          sizeof(float) * w.N, rows, cudaMemcpyDeviceToDevice, c->stream);
        if (e != cudaSuccess) rc = cuda_fail(e, "strided output copy");
    }
    if (rc == OK && host) {
        cudaError_t e = cudaMemcpyAsync(y, dyout, yout * sizeof(float), cudaMemcpyDeviceToHost, c->stream);
        if (e != cudaSuccess) rc = cuda_fail(e, "copy result");
        if (rc == OK) rc = check_device_error(c);
    }
    if (tmp || qa_tmp || out_tmp) {
        cudaStreamSynchronize(c->stream);
        if (tmp) cudaFree(tmp);
        if (qa_tmp) { cudaFree(qa_tmp); cudaFree(da_tmp); }
        if (out_tmp) cudaFree(out_tmp);
    }
    return rc;
}

int laya_q8_0_linear(laya_ctx* c, const char* weight, const float* x, int rows, int input_stride, const float* bias,
                     float* y, int output_stride) {
    return q8_linear_impl(c, weight, x, rows, input_stride, bias, y, output_stride, true);
}
int laya_q8_0_linear_device(laya_ctx* c, const char* weight, const float* x, int rows, int input_stride,
                            const float* bias, float* y, int output_stride) {
    return q8_linear_impl(c, weight, x, rows, input_stride, bias, y, output_stride, false);
}

int laya_gemm_bf16_device(laya_ctx* c, int M, int N, int K, const uint16_t* A, int lda, int a_mn, const uint16_t* B,
                          int ldb, int b_mn, const float* bias, int epilogue, void* out, int ldo) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    if (epilogue < 0 || epilogue > 2) { set_error("unknown epilogue"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    bf::Args a{};
    a.M = M; a.N = N; a.K = K;
    a.A = reinterpret_cast<const __nv_bfloat16*>(A); a.lda = lda; a.a_mn = a_mn != 0;
    a.B = reinterpret_cast<const __nv_bfloat16*>(B); a.ldb = ldb; a.b_mn = b_mn != 0;
    a.bias = bias; a.epi = epilogue; a.out = out; a.ldo = ldo; a.err = c->err;
    a.ksplit_ok = epilogue == 2;
    return bf::gemm(a, c->stream);
}

int laya_gemm_bf16_split_device(laya_ctx* c, int M, int N, int K, const uint16_t* A, const uint16_t* A_lo, int lda,
                                int a_mn, const uint16_t* B, const uint16_t* B_lo, int ldb, int b_mn, const float* bias,
                                int epilogue, void* out, int ldo) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    if (!A_lo) { set_error("split product needs the low part of A"); return ERR_ARGUMENT; }
    if (epilogue < 0 || epilogue > 2) { set_error("unknown epilogue"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    bf::Args a{};
    a.M = M; a.N = N; a.K = K;
    a.A = reinterpret_cast<const __nv_bfloat16*>(A); a.lda = lda; a.a_mn = a_mn != 0;
    a.B = reinterpret_cast<const __nv_bfloat16*>(B); a.ldb = ldb; a.b_mn = b_mn != 0;
    a.A2 = reinterpret_cast<const __nv_bfloat16*>(A_lo); a.B2 = reinterpret_cast<const __nv_bfloat16*>(B_lo);
    a.bias = bias; a.epi = epilogue; a.out = out; a.ldo = ldo; a.err = c->err;
    a.ksplit_ok = epilogue == 2;
    return bf::gemm(a, c->stream);
}

// ------------------------------------------------------------------------------------------------ forward
int laya_decision_forward(laya_ctx* c, const int32_t* ids, const int32_t* seg_len, const int32_t* qtype, int n_items,
                          const int32_t* marker_count, const int32_t* markers, float* logits, float* act_probs) {
    if (!c || (n_items > 0 && (!ids || !seg_len || !qtype || !marker_count))) { set_error("invalid argument"); return ERR_ARGUMENT; }
    if (n_items == 0) return OK;
    DeviceGuard g(c->device);
    long long T, M;
    RC(stage_inputs(c, ids, seg_len, qtype, n_items, marker_count, markers, &T, &M));
    RC(forward_staged(c, n_items, static_cast<int>(T), static_cast<int>(M), c->logits, act_probs ? c->act : nullptr, false));
    if (M > 0 && logits) LAYA_CUDA(cudaMemcpyAsync(logits, c->logits, sizeof(float) * M, cudaMemcpyDeviceToHost, c->stream));
    if (act_probs) LAYA_CUDA(cudaMemcpyAsync(act_probs, c->act, sizeof(float) * n_items * c->d.n_act, cudaMemcpyDeviceToHost, c->stream));
    return check_device_error(c);
}

int laya_decision_forward_device(laya_ctx* c, const int32_t* ids, const int32_t* seg_len, const int32_t* qtype,
                                 int n_items, int n_tokens, const int32_t* marker_count, const int32_t* markers,
                                 int n_markers, float* logits, float* act_probs) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    if (n_items == 0) return OK;
    DeviceGuard g(c->device);
    RC(check_forward_args(c, n_items, n_tokens, n_markers));
    LAYA_CUDA(cudaMemcpyAsync(c->ids, ids, sizeof(int32_t) * n_tokens, cudaMemcpyDeviceToDevice, c->stream));
    LAYA_CUDA(cudaMemcpyAsync(c->seg_len, seg_len, sizeof(int32_t) * n_items, cudaMemcpyDeviceToDevice, c->stream));
    LAYA_CUDA(cudaMemcpyAsync(c->qtype, qtype, sizeof(int32_t) * n_items, cudaMemcpyDeviceToDevice, c->stream));
    LAYA_CUDA(cudaMemcpyAsync(c->mk_count, marker_count, sizeof(int32_t) * n_items, cudaMemcpyDeviceToDevice, c->stream));
    if (n_markers > 0) LAYA_CUDA(cudaMemcpyAsync(c->markers, markers, sizeof(int32_t) * n_markers, cudaMemcpyDeviceToDevice, c->stream));
    return forward_staged(c, n_items, n_tokens, n_markers, logits, act_probs, false);
}

int laya_encoder_forward(laya_ctx* c, const int32_t* ids, const int32_t* seg_len, int n_items, float* hidden) {
    if (!c || (n_items > 0 && (!ids || !seg_len || !hidden))) { set_error("invalid argument"); return ERR_ARGUMENT; }
    if (n_items == 0) return OK;
    DeviceGuard g(c->device);
    long long T, M;
    RC(stage_inputs(c, ids, seg_len, nullptr, n_items, nullptr, nullptr, &T, &M));
    RC(forward_staged(c, n_items, static_cast<int>(T), 0, nullptr, nullptr, true));
    LAYA_CUDA(cudaMemcpyAsync(hidden, c->h, sizeof(float) * T * c->d.hidden, cudaMemcpyDeviceToHost, c->stream));
    return check_device_error(c);
}

int laya_encoder_layer(laya_ctx* c, int layer, float* hidden, const int32_t* seg_len, int n_items) {
    if (!c || !hidden || !seg_len || n_items <= 0) { set_error("invalid argument"); return ERR_ARGUMENT; }
    if (layer < 0 || layer >= c->d.layers) { set_error("no such layer"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    long long T = 0;
    for (int i = 0; i < n_items; ++i) T += seg_len[i];
    RC(check_forward_args(c, n_items, T, 0));
    LAYA_CUDA(cudaMemcpyAsync(c->seg_len, seg_len, sizeof(int32_t) * n_items, cudaMemcpyHostToDevice, c->stream));
    LAYA_CUDA(cudaMemsetAsync(c->mk_count, 0, sizeof(int32_t) * n_items, c->stream));
    LAYA_CUDA(cudaMemcpyAsync(c->h, hidden, sizeof(float) * T * c->d.hidden, cudaMemcpyHostToDevice, c->stream));
    RC(run_plan(c, n_items, static_cast<int>(T), 0));
    RC(encoder_layer(c, layer, static_cast<int>(T)));
    LAYA_CUDA(cudaMemcpyAsync(hidden, c->h, sizeof(float) * T * c->d.hidden, cudaMemcpyDeviceToHost, c->stream));
    return check_device_error(c);
}

int laya_record_enable(laya_ctx* c, int enabled) {
    if (!c) { set_error("null context"); return ERR_ARGUMENT; }
    c->record = enabled != 0;
    return OK;
}

int laya_record_get(laya_ctx* c, const char* name, float* host, int64_t count) {
    if (!c || !name || !host) { set_error("invalid argument"); return ERR_ARGUMENT; }
    DeviceGuard g(c->device);
    auto it = c->rec.find(name);
    if (it == c->rec.end()) { set_error(std::string("nothing recorded under ") + name); return ERR_NOT_FOUND; }
    const int64_t have = static_cast<int64_t>(it->second.bytes / sizeof(float));
    LAYA_CUDA(cudaStreamSynchronize(c->stream));
    LAYA_CUDA(cudaMemcpy(host, it->second.p, sizeof(float) * std::min(have, count), cudaMemcpyDeviceToHost));
    return OK;
}

}  // extern "C"
