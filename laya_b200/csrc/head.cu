// head.cu — per-forward planning and the decision readout.
//
//   plan         segment offsets, marker offsets and the 64-query tile table of the attention kernel, from the
//                per-question lengths (DecisionModel.Forward's segment building, Laya/Models/DecisionModel.cs:133-142)
//   tokens       token -> question map (for the type embedding) and marker -> row map, with bounds checks
//   scorer       DecisionModel.ReadOut's scorer (DecisionModel.cs:178-186): LayerNorm(+bias, 1e-5) → Linear → GELU → Linear
//   act head     DecisionModel.ReadOut's calibration features + act head (DecisionModel.cs:189-228)
// The scorer and act head are tiny; they follow SimdOps.Dot's two-accumulator lane order (SimdOps.cs:64-85) and
// SimdOps.LayerNorm's, so their outputs match the CPU restatement bit for bit given the same inputs.
#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace laya {

// ------------------------------------------------------------------------------------------------ helpers
// SimdOps.Dot: 8-lane accumulators s0 (elements i..i+7) and s1 (i+8..i+15) per 16-element step with FMA, one more
// 8-lane step into s0, horizontal sums, then a scalar multiply-add tail.
DEVI float hsum8(const float* a) {
    float lo0 = __fadd_rn(a[0], a[4]), lo1 = __fadd_rn(a[1], a[5]);
    float lo2 = __fadd_rn(a[2], a[6]), lo3 = __fadd_rn(a[3], a[7]);
    return __fadd_rn(__fadd_rn(lo0, lo1), __fadd_rn(lo2, lo3));
}
DEVI float ref_dot(const float* a, const float* b, int n) {
    float s0[8], s1[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) s0[l] = s1[l] = 0.0f;
    int i = 0;
    for (; i <= n - 16; i += 16) {
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            s0[l] = __fmaf_rn(a[i + l], b[i + l], s0[l]);
            s1[l] = __fmaf_rn(a[i + 8 + l], b[i + 8 + l], s1[l]);
        }
    }
    for (; i <= n - 8; i += 8) {
#pragma unroll
        for (int l = 0; l < 8; ++l) s0[l] = __fmaf_rn(a[i + l], b[i + l], s0[l]);
    }
    float sum = __fadd_rn(hsum8(s0), hsum8(s1));
    for (; i < n; ++i) sum = __fadd_rn(sum, __fmul_rn(a[i], b[i]));
    return sum;
}

// SimdOps.LayerNorm on one row by one thread, in the reference's lane order (n a multiple of 8 here).
DEVI void ref_layer_norm(const float* x, int n, const float* w, const float* b, float eps, float* out) {
    float acc[8];
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
    for (int i = 0; i < n; i += 8)
#pragma unroll
        for (int l = 0; l < 8; ++l) acc[l] = __fadd_rn(acc[l], x[i + l]);
    const float mean = __fdiv_rn(hsum8(acc), static_cast<float>(n));
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[l] = 0.0f;
    for (int i = 0; i < n; i += 8)
#pragma unroll
        for (int l = 0; l < 8; ++l) { const float d = __fsub_rn(x[i + l], mean); acc[l] = __fmaf_rn(d, d, acc[l]); }
    const float var = __fdiv_rn(hsum8(acc), static_cast<float>(n));
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    for (int i = 0; i < n; ++i) {
        float y = __fmul_rn(__fmul_rn(__fsub_rn(x[i], mean), inv), w[i]);
        out[i] = b ? __fadd_rn(y, b[i]) : y;
    }
}

// ------------------------------------------------------------------------------------------------ plan
// Exclusive block-wide scan of v[0..n) into out[0..n); returns the total (every thread).
// transform_tiles: count ⌈v / transform_tiles⌉ (tiles of that many rows) instead of v.
DEVI int block_scan(const int32_t* v, int n, int32_t* out, int* sh, int transform_tiles) {
    const int tid = threadIdx.x, nt = blockDim.x;
    const int per = (n + nt - 1) / nt;
    const int lo = min(n, tid * per), hi = min(n, lo + per);
    const int tt = transform_tiles;
    int local = 0;
    for (int i = lo; i < hi; ++i) local += tt ? (v[i] + tt - 1) / tt : v[i];
    sh[tid] = local;
    __syncthreads();
    for (int off = 1; off < nt; off <<= 1) {
        int add = tid >= off ? sh[tid - off] : 0;
        __syncthreads();
        sh[tid] += add;
        __syncthreads();
    }
    int run = sh[tid] - local;
    const int total = sh[nt - 1];
    for (int i = lo; i < hi; ++i) { out[i] = run; run += tt ? (v[i] + tt - 1) / tt : v[i]; }
    __syncthreads();
    return total;
}

__global__ void __launch_bounds__(1024) plan_kernel(PlanArgs a) {
    __shared__ int sh[1024];
    const int n = a.n_items;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        if (a.seg_len[i] < 0 || a.marker_count[i] < 0) atomicExch(a.err, LAYA_DEV_ERR_BOUNDS);
    const int tokens = block_scan(a.seg_len, n, a.seg_start, sh, 0);
    const int markers = block_scan(a.marker_count, n, a.mk_start, sh, 0);
    const int tiles = block_scan(a.seg_len, n, a.qt_start, sh, 64);
    if (threadIdx.x == 0) {
        if (tokens != a.n_tokens || markers != a.n_markers || tiles > a.max_qtiles) atomicExch(a.err, LAYA_DEV_ERR_BOUNDS);
        *a.n_qtiles = min(tiles, a.max_qtiles);
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int t0 = a.qt_start[i], nt = (a.seg_len[i] + 63) / 64;
        for (int j = 0; j < nt; ++j)
            if (t0 + j < a.max_qtiles) { a.qt_item[t0 + j] = i; a.qt_q0[t0 + j] = 64 * j; }
    }
    if (!a.tq_start) return;
    const int tiles128 = block_scan(a.seg_len, n, a.tq_start, sh, 128);
    if (threadIdx.x == 0) {
        if (tiles128 > a.max_tq) atomicExch(a.err, LAYA_DEV_ERR_BOUNDS);
        *a.n_tq = min(tiles128, a.max_tq);
    }
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int t0 = a.tq_start[i], nt = (a.seg_len[i] + 127) / 128;
        for (int j = 0; j < nt; ++j)
            if (t0 + j < a.max_tq) { a.tq_item[t0 + j] = i; a.tq_p0[t0 + j] = 128 * j; }
    }
}

DEVI int upper_bound_idx(const int32_t* starts, int n, int x) {   // last i with starts[i] <= x
    int lo = 0, hi = n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (starts[mid] <= x) lo = mid; else hi = mid - 1;
    }
    return lo;
}

__global__ void tokens_kernel(PlanArgs a) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < a.n_tokens) a.tok_item[i] = upper_bound_idx(a.seg_start, a.n_items, i);
    if (i < a.n_markers) {
        const int it = upper_bound_idx(a.mk_start, a.n_items, i);
        // skip questions with no markers: the last item whose start is <= i and that has markers
        int item = it;
        while (item > 0 && a.marker_count[item] == 0) --item;
        int pos = a.markers[i];
        pos = pos < 0 ? 0 : pos;
        if (pos >= a.seg_len[item]) { atomicExch(a.err, LAYA_DEV_ERR_BOUNDS); pos = 0; }
        a.marker_row[i] = a.seg_start[item] + pos;
        a.marker_item[i] = item;
    }
}

int plan(const PlanArgs& a, cudaStream_t stream) {
    plan_kernel<<<1, 1024, 0, stream>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    const int n = a.n_tokens > a.n_markers ? a.n_tokens : a.n_markers;
    if (n > 0) {
        tokens_kernel<<<(n + 255) / 256, 256, 0, stream>>>(a);
        count_launch();
        LAYA_CUDA(cudaGetLastError());
    }
    return OK;
}

// ------------------------------------------------------------------------------------------------ scorer
// SimdOps.Dot's 16 accumulation chains (element i goes to chain i mod 16) by a half-warp, one chain per lane with
// coalesced loads, combined in the reference's order: octet sums of s0 (lanes 0-7) and s1 (lanes 8-15), then s0 + s1.
// n must be a multiple of 16 (the scorer's hidden size).  Every lane of the half-warp returns the dot.
DEVI float halfwarp_ref_dot(const float* a, const float* b, int n, int l16) {
    float acc = 0.0f;
    for (int i = l16; i < n; i += 16) acc = __fmaf_rn(a[i], b[i], acc);
    // hsum8 of the octet: (a0+a4, a1+a5, a2+a6, a3+a7) then pairwise, as octet_hsum in norm.cu
    float t = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
    float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
    float v = __fadd_rn(u, __shfl_xor_sync(0xffffffffu, u, 2));
    const float other = __shfl_xor_sync(0xffffffffu, v, 8);   // the other octet's sum
    return l16 < 8 ? __fadd_rn(v, other) : __fadd_rn(other, v);
}

constexpr int SC_MK = 8;     // markers per CTA
constexpr int SC_OUT = 128;  // Linear1 outputs per CTA

// grid (marker groups, output chunks): LayerNorm of the CTA's marker rows, then SC_OUT outputs of
// GELU(Linear1) for each of them, each weight row read once per CTA.
__global__ void __launch_bounds__(256) scorer_hidden_kernel(ScorerArgs a) {
    extern __shared__ float sm[];
    const int H = a.hidden;
    float* xs = sm;   // [SC_MK][H]
    const int m0 = blockIdx.x * SC_MK;
    const int nm = min(SC_MK, a.n_markers - m0);
    if (threadIdx.x < nm) {
        const float* row = a.h + static_cast<size_t>(a.marker_row[m0 + threadIdx.x]) * H;
        ref_layer_norm(row, H, a.ln_w, a.ln_b, 1e-5f, xs + threadIdx.x * H);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, half = (threadIdx.x >> 4) & 1, l16 = threadIdx.x & 15;
    const int j0 = blockIdx.y * SC_OUT, jend = min(H, j0 + SC_OUT);
    // warp-uniform trip count (the shuffles need all 32 lanes): the second half-warp repeats row jj past the end
    for (int jj = j0 + 2 * warp; jj < jend; jj += 16) {
        const int j = jj + half;
        const bool valid = j < jend;
        const float* wj = a.w1 + static_cast<size_t>(valid ? j : jj) * H;
        for (int m = 0; m < nm; ++m) {
            const float d = halfwarp_ref_dot(xs + m * H, wj, H, l16);
            if (valid && l16 == 0) a.hid[static_cast<size_t>(m0 + m) * H + j] = ref_gelu(__fadd_rn(d, a.b1[j]));
        }
    }
}

// logit = Dot(hidden, w2) + b2: one half-warp per marker.
__global__ void __launch_bounds__(256) scorer_logit_kernel(ScorerArgs a) {
    const int hw = (blockIdx.x * blockDim.x + threadIdx.x) >> 4, l16 = threadIdx.x & 15;
    const int m = hw < a.n_markers ? hw : a.n_markers - 1;
    const float d = halfwarp_ref_dot(a.hid + static_cast<size_t>(m) * a.hidden, a.w2, a.hidden, l16);
    if (hw < a.n_markers && l16 == 0) a.logits[m] = __fadd_rn(d, a.b2[0]);
}

// SimdOps.Softmax (SimdOps.cs:275-291) by one thread.
DEVI void ref_softmax(float* v, int n) {
    if (n <= 0) return;
    float mx = v[0];
    for (int i = 1; i < n; ++i) mx = fmaxf(mx, v[i]);
    if (mx == -INFINITY) { for (int i = 0; i < n; ++i) v[i] = 0.0f; return; }
    float total = 0.0f;
    for (int i = 0; i < n; ++i) { const float e = expf(__fsub_rn(v[i], mx)); v[i] = e; total = __fadd_rn(total, e); }
    const float s = total > 0.0f ? __fdiv_rn(1.0f, total) : 0.0f;
    for (int i = 0; i < n; ++i) v[i] = __fmul_rn(v[i], s);
}

__global__ void __launch_bounds__(256) act_kernel(ActArgs a) {
    extern __shared__ float sm[];
    const int H = a.hidden, item = blockIdx.x;
    float* in = sm;                       // [H + 4]
    float* a1 = sm + H + 8;               // [act_hidden]
    float* a2 = a1 + a.act_hidden;        // [n_act]
    float* p = a2 + a.n_act + 4;          // [k] probabilities (k <= max_markers_per_item)
    const int k = a.marker_count[item];
    const int mk0 = a.mk_start[item];
    const float* pooled = a.h + static_cast<size_t>(a.seg_start[item]) * H;
    for (int i = threadIdx.x; i < H; i += blockDim.x) in[i] = pooled[i];
    if (threadIdx.x == 0) {
        for (int i = 0; i < k; ++i) p[i] = a.logits[mk0 + i];
        ref_softmax(p, k);
        const float kk = static_cast<float>(k > 2 ? k : 2);
        float ent = 0.0f;
        for (int i = 0; i < k; ++i) ent = __fsub_rn(ent, __fmul_rn(p[i], logf(fminf(fmaxf(p[i], 1e-9f), 3.40282347e38f))));
        ent = __fdiv_rn(ent, logf(kk));
        float top1 = 0.0f, top2 = 0.0f;
        for (int i = 0; i < k; ++i) {
            if (p[i] > top1) { top2 = top1; top1 = p[i]; }
            else if (p[i] > top2) top2 = p[i];
        }
        in[H] = top1;
        in[H + 1] = __fsub_rn(top1, top2);
        in[H + 2] = ent;
        in[H + 3] = __fdiv_rn(kk, 255.0f);
    }
    __syncthreads();
    for (int j = threadIdx.x; j < a.act_hidden; j += blockDim.x)
        a1[j] = ref_gelu(__fadd_rn(ref_dot(in, a.w1 + static_cast<size_t>(j) * (H + 4), H + 4), a.b1[j]));
    __syncthreads();
    for (int j = threadIdx.x; j < a.n_act; j += blockDim.x)
        a2[j] = __fadd_rn(ref_dot(a1, a.w2 + static_cast<size_t>(j) * a.act_hidden, a.act_hidden), a.b2[j]);
    __syncthreads();
    if (threadIdx.x == 0) {
        ref_softmax(a2, a.n_act);
        for (int j = 0; j < a.n_act; ++j) a.probs[static_cast<size_t>(item) * a.n_act + j] = a2[j];
    }
}

int scorer(const ScorerArgs& a, cudaStream_t stream) {
    if (a.n_markers <= 0) return OK;
    if (a.hidden % 16) { set_error("scorer hidden size must be a multiple of 16"); return ERR_NOT_SUPPORTED; }
    const size_t smem = sizeof(float) * SC_MK * a.hidden;
    if (smem > 48 * 1024)
        LAYA_CUDA(cudaFuncSetAttribute(scorer_hidden_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    dim3 grid((a.n_markers + SC_MK - 1) / SC_MK, (a.hidden + SC_OUT - 1) / SC_OUT);
    scorer_hidden_kernel<<<grid, 256, smem, stream>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    scorer_logit_kernel<<<(a.n_markers * 16 + 255) / 256, 256, 0, stream>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

int act_head(const ActArgs& a, cudaStream_t stream) {
    if (a.n_items <= 0) return OK;
    const size_t smem = sizeof(float) * (a.hidden + 8 + a.act_hidden + a.n_act + 4 + a.max_k);
    act_kernel<<<a.n_items, 256, smem, stream>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace laya
