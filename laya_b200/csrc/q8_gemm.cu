// q8_gemm.cu — the Q8_0 product on sm_100a tensor cores.
//
// Replaces PackedMatrixQ8_0.Multiply/Run/Panel512 (Base/Numerics/PackedMatrixQ8_0.cs:224-557) and the two
// quantizers of Q8_0 (PackedMatrixQ8_0.cs:20-71).
//
// Definition being computed (PackedMatrixQ8_0Tests.cs:145-182):
//     out[r, c] = bias[c];  for b in 0 .. K/32-1:  out[r, c] = fma((float)Σ_b, d_w[c, b] · d_x[r, b], out[r, c])
// with Σ_b = Σ_{k in block b} q_x[r, k] · q_w[c, k] an exact int32.
//
// One Q8_0 block (32 int8 along K) is exactly one tcgen05.mma.kind::i8 instruction (K = 32).  Every block's
// product goes to its own TMEM accumulator (the instruction overwrites, it never accumulates), so the exact
// int32 block sums Σ_b land in TMEM one block at a time.  Epilogue warps drain them with tcgen05.ld and apply
// the reference's rescale in the reference's order, keeping the fp32 accumulators in registers; the result
// is therefore bit-identical to the definition above.
//
// CTA layout (one CTA per SM; 128 × BN output tile):
//   warp 0      TMA producer: A (activation codes, 128 rows × 128 B) and B (weight codes, BN rows × 128 B)
//               per stage, 128-byte swizzle, STAGES-deep ring.
//   warp 1      TMEM allocator + MMA issuer (one thread): 4 MMAs per stage, one per Q8_0 block, each into
//               TMEM buffer (block mod NBUF), committed to that buffer's "full" barrier.
//   warps 2..   EPI_WARPS epilogue warps.  tcgen05.ld restricts warp w to TMEM lanes 32·(w mod 4)…+31, so the
//               warps split as 4 lane quarters × (EPI_WARPS/4) column groups; a thread owns one output row
//               and CPT consecutive columns.
// The per-block rescale (cvt + mul + fma per output per block) is the throughput bound, not the MMA.
#include "common.cuh"
#include "internal.h"

namespace laya {
namespace q8 {

constexpr int BM = 128;        // tile rows (tokens)
constexpr int BK = 128;        // K bytes per stage = 4 Q8_0 blocks
constexpr int BPS = BK / 32;   // blocks per stage

template <int BN, int EPI_WARPS, int STAGES>
struct Cfg {
    static constexpr int A_BYTES = BM * BK;
    static constexpr int B_BYTES = BN * BK;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int NBUF = (512 / BN) < 4 ? (512 / BN) : 4;
    static constexpr int GROUPS = EPI_WARPS / 4;
    static constexpr int CPT = BN / GROUPS;
    static constexpr int THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int BAR_BYTES = 8 * (2 * STAGES + 2 * NBUF) + 16;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
    static_assert(CPT % 32 == 0, "each epilogue thread owns whole 32-column TMEM loads");
    static_assert(EPI_WARPS % 4 == 0, "epilogue warps come in lane-quarter sets");
};

struct KParams {
    int M, N, K;
    const float* dx; int ldx;
    const float* dw; int ldw;
    const float* bias;
    float* out; int ldo;
    int8_t* qout; int ldqo;
    float* qsc; int ldqs;
    int* err;
};

// Quantizes 32 consecutive fp32 values held by one thread to Q8_0 (Q8_0.QuantizeActivations,
// PackedMatrixQ8_0.cs:50-71): d = amax/127 stored fp16, id = 127/amax, q = round-half-even(x · id).
DEVI void quantize_block32_store(const float* v, int8_t* qdst, float* ddst) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    uint32_t packed[8];
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        uint32_t word = 0;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            int qi = __float2int_rn(__fmul_rn(v[w * 4 + t], id));
            word |= (static_cast<uint32_t>(qi) & 0xFFu) << (8 * t);
        }
        packed[w] = word;
    }
    uint4* q4 = reinterpret_cast<uint4*>(qdst);
    q4[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    q4[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    *ddst = round_fp16(d);
}

template <int BN, int EPI_WARPS, int STAGES, int EPI>
__global__ void __launch_bounds__(Cfg<BN, EPI_WARPS, STAGES>::THREADS, 1)
    q8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, KParams p) {
    using C = Cfg<BN, EPI_WARPS, STAGES>;
    constexpr int NBUF = C::NBUF;
    constexpr int CPT = C::CPT;
    constexpr uint32_t IDESC = make_idesc(/*D s32*/ 2, /*A s8*/ 1, /*B s8*/ 1, BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + NBUF;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + NBUF);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = warp_id(), lane = lane_id();
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int nblk = p.K / 32;
    const int iters = (nblk + BPS - 1) / BPS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
        for (int b = 0; b < NBUF; ++b) { mbar_init(tfull + b, 1); mbar_init(tempty + b, EPI_WARPS); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tmA); prefetch_tmap(&tmB); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            for (int it = 0; it < iters; ++it) {
                const int s = it % STAGES;
                if (!mbar_wait(empty + s, ((it / STAGES) & 1) ^ 1, abort_flag, p.err)) break;
                mbar_arrive_expect_tx(full + s, C::STAGE_BYTES);
                tma_load_2d(sA + s * C::A_BYTES, &tmA, full + s, it * BK, m0);
                tma_load_2d(sB + s * C::B_BYTES, &tmB, full + s, it * BK, n0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int b = 0; b < nblk; ++b) {
                const int it = b / BPS, j = b % BPS, s = it % STAGES;
                if (j == 0) {
                    if (!mbar_wait(full + s, (it / STAGES) & 1, abort_flag, p.err)) break;
                    tc_fence_after();
                }
                const int buf = b % NBUF;
                if (!mbar_wait(tempty + buf, ((b / NBUF) & 1) ^ 1, abort_flag, p.err)) break;
                tc_fence_after();
                const uint64_t ad = smem_desc_sw128(smem_u32(sA + s * C::A_BYTES + j * 32));
                const uint64_t bd = smem_desc_sw128(smem_u32(sB + s * C::B_BYTES + j * 32));
                mma_i8(tmem + static_cast<uint32_t>(buf * BN), ad, bd, IDESC, 0u);
                mma_commit(tfull + buf);
                if (j == BPS - 1 || b == nblk - 1) mma_commit(empty + s);
            }
        }
    } else {
        // ------------------------------------------------------------------ epilogue warps
        const int e = warp - 2;
        const int quarter = warp & 3;
        const int grp = e >> 2;
        const int row = quarter * 32 + lane;
        const int grow = m0 + row;
        const int col0 = grp * CPT;
        const int gcol0 = n0 + col0;

        float acc[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
            const int c = gcol0 + j;
            acc[j] = (p.bias != nullptr && c < p.N) ? __ldg(p.bias + c) : 0.0f;
        }
        const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(col0);
        const float* dxp = p.dx + grow;
        bool ok = true;
        float dxr = __ldg(dxp);
        for (int b = 0; b < nblk; ++b) {
            const int buf = b % NBUF;
            const float dx_next = (b + 1 < nblk) ? __ldg(dxp + static_cast<size_t>(b + 1) * p.ldx) : 0.0f;
            const float4* dwp = reinterpret_cast<const float4*>(p.dw + static_cast<size_t>(b) * p.ldw + gcol0);
            if (!mbar_wait(tfull + buf, (b / NBUF) & 1, abort_flag, p.err)) { ok = false; break; }
            tc_fence_after();
            uint32_t s[CPT / 32][32];
#pragma unroll
            for (int c = 0; c < CPT / 32; ++c) tmem_ld32(tbase + static_cast<uint32_t>(buf * BN + c * 32), s[c]);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty + buf);
#pragma unroll
            for (int j4 = 0; j4 < CPT / 4; ++j4) {
                const float4 w = __ldg(dwp + j4);
                const int j = j4 * 4;
                acc[j + 0] = __fmaf_rn(i2f_exact(static_cast<int32_t>(s[(j + 0) / 32][(j + 0) % 32])), __fmul_rn(w.x, dxr), acc[j + 0]);
                acc[j + 1] = __fmaf_rn(i2f_exact(static_cast<int32_t>(s[(j + 1) / 32][(j + 1) % 32])), __fmul_rn(w.y, dxr), acc[j + 1]);
                acc[j + 2] = __fmaf_rn(i2f_exact(static_cast<int32_t>(s[(j + 2) / 32][(j + 2) % 32])), __fmul_rn(w.z, dxr), acc[j + 2]);
                acc[j + 3] = __fmaf_rn(i2f_exact(static_cast<int32_t>(s[(j + 3) / 32][(j + 3) % 32])), __fmul_rn(w.w, dxr), acc[j + 3]);
            }
            dxr = dx_next;
        }

        if (ok && grow < p.M) {
            if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
                float* o = p.out + static_cast<size_t>(grow) * p.ldo + gcol0;
                const bool vec = (gcol0 + CPT <= p.N) && ((p.ldo & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.out) & 15) == 0);
                if (vec) {
#pragma unroll
                    for (int j4 = 0; j4 < CPT / 4; ++j4) {
                        float4 v = make_float4(acc[4 * j4], acc[4 * j4 + 1], acc[4 * j4 + 2], acc[4 * j4 + 3]);
                        float4* dst = reinterpret_cast<float4*>(o) + j4;
                        if constexpr (EPI == EPI_RESID) {
                            const float4 h = *dst;
                            v.x = __fadd_rn(h.x, v.x); v.y = __fadd_rn(h.y, v.y);
                            v.z = __fadd_rn(h.z, v.z); v.w = __fadd_rn(h.w, v.w);
                        }
                        *dst = v;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < CPT; ++j) {
                        if (gcol0 + j < p.N) {
                            if constexpr (EPI == EPI_RESID) o[j] = __fadd_rn(o[j], acc[j]);
                            else o[j] = acc[j];
                        }
                    }
                }
            } else if constexpr (EPI == EPI_GEGLU_Q8) {
                // Column groups of 64: [32 GELU inputs | their 32 gates] -> 32 activations = one Q8_0 block of
                // the next product's input (ModernBertEncoder.GeGlu, ModernBertEncoder.cs:204-214).
#pragma unroll
                for (int g = 0; g < CPT / 64; ++g) {
                    const int pcol = gcol0 + g * 64;
                    if (pcol < p.N) {
                        const int blk = pcol / 64;
                        float act[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) act[j] = __fmul_rn(ref_gelu(acc[g * 64 + j]), acc[g * 64 + 32 + j]);
                        quantize_block32_store(act, p.qout + static_cast<size_t>(grow) * p.ldqo + blk * 32,
                                               p.qsc + static_cast<size_t>(blk) * p.ldqs + grow);
                    }
                }
            } else if constexpr (EPI == EPI_RELU_Q8) {
                // nn.TransformerEncoderLayer's ReLU feed-forward (DecisionModel.cs:300), quantized for linear2.
#pragma unroll
                for (int g = 0; g < CPT / 32; ++g) {
                    const int c = gcol0 + g * 32;
                    if (c < p.N) {
                        float act[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) act[j] = fmaxf(acc[g * 32 + j], 0.0f);
                        quantize_block32_store(act, p.qout + static_cast<size_t>(grow) * p.ldqo + c,
                                               p.qsc + static_cast<size_t>(c / 32) * p.ldqs + grow);
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ------------------------------------------------------------------------------------------------ host

template <int BN, int EPI_WARPS, int STAGES, int EPI>
static int launch(const GemmArgs& a, cudaStream_t stream) {
    using C = Cfg<BN, EPI_WARPS, STAGES>;
    CUtensorMap tA, tB;
    int rc = make_tmap_2d(&tA, a.qx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.M, a.K, a.K, BM, BK);
    if (rc) return rc;
    rc = make_tmap_2d(&tB, a.qw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, a.N, a.K, a.K, BN, BK);
    if (rc) return rc;
    auto kern = q8_gemm_kernel<BN, EPI_WARPS, STAGES, EPI>;
    static bool attr_set = false;   // per instantiation
    if (!attr_set) {
        LAYA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_set = true;
    }
    KParams p{a.M, a.N, a.K, a.dx, a.ldx, a.dw, a.ldw, a.bias, a.out, a.ldo, a.qout, a.ldqo, a.qsc, a.ldqs, a.err};
    dim3 grid((a.N + BN - 1) / BN, (a.M + BM - 1) / BM);
    kern<<<grid, C::THREADS, C::SMEM, stream>>>(tA, tB, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

int gemm(const GemmArgs& a, cudaStream_t stream) {
    if (a.M <= 0 || a.N <= 0) return OK;
    if (a.K <= 0 || a.K % 32 != 0) { set_error("Q8_0 needs a multiple of 32 inputs"); return ERR_ARGUMENT; }
    if (a.ldx < ((a.M + BM - 1) / BM) * BM) { set_error("activation scale stride below the padded row count"); return ERR_ARGUMENT; }
    if (a.ldw < ((a.N + 127) / 128) * 128) { set_error("weight scale stride below the padded column count"); return ERR_ARGUMENT; }
    if ((reinterpret_cast<uintptr_t>(a.qx) & 15) || (reinterpret_cast<uintptr_t>(a.qw) & 15)) {
        set_error("Q8_0 operands must be 16-byte aligned"); return ERR_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(a.dw) & 15) || (a.ldw & 3)) { set_error("weight scales must be 16-byte aligned rows"); return ERR_ARGUMENT; }
    constexpr int BN = 128, EW = 8, ST = 4;
    switch (a.epi) {
        case EPI_STORE: return launch<BN, EW, ST, EPI_STORE>(a, stream);
        case EPI_RESID: return launch<BN, EW, ST, EPI_RESID>(a, stream);
        case EPI_GEGLU_Q8:
            if (a.N % 64) { set_error("GeGLU product needs whole 64-column groups"); return ERR_ARGUMENT; }
            return launch<BN, EW, ST, EPI_GEGLU_Q8>(a, stream);
        case EPI_RELU_Q8:
            if (a.N % 32) { set_error("ReLU product needs whole 32-column blocks"); return ERR_ARGUMENT; }
            return launch<BN, EW, ST, EPI_RELU_Q8>(a, stream);
    }
    set_error("unknown epilogue");
    return ERR_ARGUMENT;
}

// ------------------------------------------------------------------------------------------------ quantizers

// One warp per 32-value block; lane j owns value j.
__global__ void quantize_activations_kernel(const float* __restrict__ x, int rows, int stride, int K,
                                            int8_t* __restrict__ q, float* __restrict__ d, int ldd) {
    const int nb = K / 32;
    const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= static_cast<long long>(rows) * nb) return;
    const int r = static_cast<int>(gw / nb), b = static_cast<int>(gw % nb);
    const float v = x[static_cast<size_t>(r) * stride + b * 32 + lane];
    const float amax = warp_max(fabsf(v));
    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    q[static_cast<size_t>(r) * K + b * 32 + lane] = static_cast<int8_t>(__float2int_rn(__fmul_rn(v, id)));
    if (lane == 0) d[static_cast<size_t>(b) * ldd + r] = round_fp16(__fdiv_rn(amax, 127.0f));
}

// Q8_0.QuantizeWeightBlock (PackedMatrixQ8_0.cs:20-28): d = amax/127, id = 1/d, q = round half away.
__global__ void quantize_weights_kernel(const float* __restrict__ w, int N, int K, int8_t* __restrict__ q,
                                        float* __restrict__ d, int ldd) {
    const int nb = K / 32;
    const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= static_cast<long long>(N) * nb) return;
    const int c = static_cast<int>(gw / nb), b = static_cast<int>(gw % nb);
    const float v = w[static_cast<size_t>(c) * K + b * 32 + lane];
    const float amax = warp_max(fabsf(v));
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
    q[static_cast<size_t>(c) * K + b * 32 + lane] = static_cast<int8_t>(roundf(__fmul_rn(v, id)));
    if (lane == 0) d[static_cast<size_t>(b) * ldd + c] = round_fp16(dd);
}

int quantize_activations(const float* x, int rows, int stride, int K, int8_t* q, float* d, int ldd,
                         cudaStream_t stream) {
    if (rows <= 0) return OK;
    if (K % 32 || stride < K) { set_error("activation rows must hold whole 32-value blocks"); return ERR_ARGUMENT; }
    const long long warps = static_cast<long long>(rows) * (K / 32);
    const int threads = 256;
    const long long blocks = (warps * 32 + threads - 1) / threads;
    quantize_activations_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(x, rows, stride, K, q, d, ldd);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

int quantize_weights(const float* w, int N, int K, int8_t* q, float* d, int ldd, cudaStream_t stream) {
    if (N <= 0) return OK;
    if (K % 32) { set_error("Q8_0 needs a multiple of 32 inputs"); return ERR_ARGUMENT; }
    const long long warps = static_cast<long long>(N) * (K / 32);
    const int threads = 256;
    const long long blocks = (warps * 32 + threads - 1) / threads;
    quantize_weights_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(w, N, K, q, d, ldd);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace q8
}  // namespace laya
