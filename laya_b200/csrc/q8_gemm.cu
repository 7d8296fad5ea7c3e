// q8_gemm.cu — the Q8_0 product on sm_100a tensor cores.
//
// Replaces PackedMatrixQ8_0.Multiply/Run/Panel512 (Base/Numerics/PackedMatrixQ8_0.cs:224-557) and the two
// quantizers of Q8_0 (PackedMatrixQ8_0.cs:20-71).
//
// Definition being computed (PackedMatrixQ8_0Tests.cs:145-182):
//     out[r, c] = bias[c];  for b in 0 .. K/32-1:  out[r, c] = fma((float)Σ_b, d_w[c, b] · d_x[r, b], out[r, c])
// with Σ_b = Σ_{k in block b} q_x[r, k] · q_w[c, k] an exact integer.
//
// Codes are held as fp16 values (the integers -127..127 are exact in fp16).  Every product of two codes is an
// integer below 2^14 and every partial sum of a 32-term block stays an integer below 2^19, so the kind::f16
// tensor-core product with fp32 accumulation computes each block's Σ_b exactly — and delivers it already as the
// fp32 value (float)Σ_b the rescale needs.  Each block is its own accumulator: two K=16 MMAs (the first
// overwriting, the second accumulating) into the TMEM buffer of that block.  Epilogue warps drain the buffers
// with tcgen05.ld and apply the reference's rescale in the reference's order (one fp32 multiply d_w·d_x and one
// fma per output per block, issued as two-column mul/fma .f32x2 instructions), keeping the fp32 accumulators in
// registers: the result is bit-identical to the definition.
//
// What bounds it: every block is a round trip — its MMAs complete, the epilogue drains its TMEM buffer, the buffer
// returns to the MMA issuer — and TMEM holds at most 512 fp32 columns of such per-block sums, i.e. about 512 cycles
// of tensor work in flight per SM.  Measured here, that round trip takes several times longer than the work it
// covers (with the epilogue reduced to the handshake alone the product still runs at only ~450 T int8-op/s), so the
// tensor pipe idles most of the time (about 15% active); the epilogue's shared-memory scale reads add to the hold
// time.  Variants that moved the scale product onto the tensor cores (a third MMA per block into a second TMEM
// buffer), spread the epilogue over 16 warps, or used 16x256b loads with a four-deep TMEM ring all measured within
// 15% of this form, slower or equal, at the decoder's and the encoder's shapes.  The exact-integer fp16 form (no
// int→fp32 conversion in the epilogue) is used rather than kind::i8.
//
// CTA layout (one CTA per SM; 128 × BN output tile):
//   warp 0      TMA producer: A (activation codes, 128 rows × 64) and B (weight codes, BN rows × 64) per stage
//               with 128-byte swizzle, STAGES-deep ring; and per stage the two blocks' scales (d_x for the tile's
//               rows, d_w for its columns) into a separate SST-slot ring released by the epilogue.
//   warp 1      TMEM allocator + MMA issuer (one thread).
//   warps 2..   EPI_WARPS epilogue warps.  tcgen05.ld restricts warp w to TMEM lanes 32·(w mod 4)…+31, so the
//               warps split as 4 lane quarters × (EPI_WARPS/4) column groups; a thread owns one output row
//               and CPT consecutive columns.
#include "common.cuh"
#include "internal.h"

namespace laya {
namespace q8 {

constexpr int BM = 128;        // tile rows (tokens)
constexpr int BKB = 128;       // K bytes per stage (one 128-byte swizzle row)
constexpr int BK = BKB / 2;    // K codes per stage = 2 Q8_0 blocks
constexpr int BPS = BK / 32;   // blocks per stage
constexpr int SST = 4;         // slots of the block-scale ring

template <int BN, int EPI_WARPS, int STAGES>
struct Cfg {
    static constexpr int A_BYTES = BM * BKB;
    static constexpr int B_BYTES = BN * BKB;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int SC_FLOATS = BPS * (BM + BN);          // one scale slot: dx [2][128], dw [2][BN]
    static constexpr int SC_BYTES = SC_FLOATS * 4;
    static constexpr int NBUF = (512 / BN) < 8 ? (512 / BN) : 8;   // TMEM accumulators (one per in-flight block)
    static constexpr int GROUPS = EPI_WARPS / 4;
    static constexpr int CPT = BN / GROUPS;
    static constexpr int THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int STAGE_OUT_BYTES = 4096;               // per epilogue warp: 32 rows x 128 B of output
    static constexpr int BAR_BYTES = 8 * (2 * STAGES + 2 * SST + 2 * NBUF) + 16;
    static constexpr int SMEM = 1024 + STAGES * STAGE_BYTES + EPI_WARPS * STAGE_OUT_BYTES + SST * SC_BYTES + BAR_BYTES;
    static_assert(SMEM <= 227 * 1024, "shared memory budget");
    static_assert(CPT % 32 == 0, "each epilogue thread owns whole 32-column TMEM loads");
    static_assert(EPI_WARPS % 4 == 0, "epilogue warps come in lane-quarter sets");
    static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 1024-byte alignment of 128-byte swizzling");
};

struct KParams {
    int M, N, K;
    const float* bias;
    float* out; int ldo;
    code_t* qout; int ldqo;
    float* qsc; int ldqs;
    int* err;
};

// Quantizes 32 consecutive fp32 values held by one thread to Q8_0 (Q8_0.QuantizeActivations,
// PackedMatrixQ8_0.cs:50-71): d = amax/127 stored fp16, id = 127/amax, q = round-half-even(x · id).
DEVI void quantize_block32_store(const float* v, code_t* qdst, float* ddst) {
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    uint4* q4 = reinterpret_cast<uint4*>(qdst);
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        uint32_t word[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const __half2 h2 = __halves2half2(__int2half_rn(__float2int_rn(__fmul_rn(v[w * 8 + 2 * t], id))),
                                              __int2half_rn(__float2int_rn(__fmul_rn(v[w * 8 + 2 * t + 1], id))));
            word[t] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        q4[w] = make_uint4(word[0], word[1], word[2], word[3]);
    }
    *ddst = round_fp16(d);
}

// One block's rescale for 32 columns whose exact block sums arrive as fp32 bits in s[]:
// acc[j] = fma((float)Σ, d_w[j] · d_x, acc[j]), two columns per .f32x2 instruction.
DEVI void rescale32(float* acc, const uint32_t (&s)[32], const float* dw, float dx) {
    const float4* w4 = reinterpret_cast<const float4*>(dw);
    const uint64_t dx2 = f2_pack(dx, dx);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 w = w4[q];
        const uint64_t a01 = f2_fma(f2_pack(__uint_as_float(s[4 * q]), __uint_as_float(s[4 * q + 1])),
                                    f2_mul(f2_pack(w.x, w.y), dx2), f2_pack(acc[4 * q], acc[4 * q + 1]));
        const uint64_t a23 = f2_fma(f2_pack(__uint_as_float(s[4 * q + 2]), __uint_as_float(s[4 * q + 3])),
                                    f2_mul(f2_pack(w.z, w.w), dx2), f2_pack(acc[4 * q + 2], acc[4 * q + 3]));
        f2_unpack(a01, acc[4 * q], acc[4 * q + 1]);
        f2_unpack(a23, acc[4 * q + 2], acc[4 * q + 3]);
    }
}

template <int BN, int EPI_WARPS, int STAGES, int EPI>
__global__ void __launch_bounds__(Cfg<BN, EPI_WARPS, STAGES>::THREADS, 1)
    q8_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmDX, const __grid_constant__ CUtensorMap tmDW,
                   const __grid_constant__ CUtensorMap tmOut, KParams p) {
    using C = Cfg<BN, EPI_WARPS, STAGES>;
    constexpr int NBUF = C::NBUF;
    constexpr int CPT = C::CPT;
    constexpr uint32_t IDESC = make_idesc(/*D f32*/ 1, /*A f16*/ 0, /*B f16*/ 0, BM, BN);

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * C::A_BYTES;
    uint8_t* sOut = smem + STAGES * C::STAGE_BYTES;                          // [EPI_WARPS][4 KB] output staging
    float* sSc = reinterpret_cast<float*>(sOut + EPI_WARPS * C::STAGE_OUT_BYTES);   // [SST][dx BPS×128 | dw BPS×BN]
    uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sSc) + SST * C::SC_BYTES);
    uint64_t* empty = full + STAGES;
    uint64_t* sfull = empty + STAGES;
    uint64_t* sempty = sfull + SST;
    uint64_t* tfull = sempty + SST;
    uint64_t* tempty = tfull + NBUF;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + NBUF);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = warp_id(), lane = lane_id();
    const int nblk = p.K / 32;
    const int iters = (nblk + BPS - 1) / BPS;
    const int tiles_n = (p.N + BN - 1) / BN;
    const int tiles = tiles_n * ((p.M + BM - 1) / BM);

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) { mbar_init(full + s, 1); mbar_init(empty + s, 1); }
        for (int s = 0; s < SST; ++s) { mbar_init(sfull + s, 1); mbar_init(sempty + s, EPI_WARPS); }
        for (int b = 0; b < NBUF; ++b) { mbar_init(tfull + b, 1); mbar_init(tempty + b, EPI_WARPS); }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA); prefetch_tmap(&tmB); prefetch_tmap(&tmDX); prefetch_tmap(&tmDW); prefetch_tmap(&tmOut);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    // Persistent: every role walks the same tile sequence (N fastest, so concurrent CTAs share activation rows in
    // L2); the stage ring, scale ring and TMEM buffers run on across tiles, so one tile's stores overlap the next
    // tile's loads and MMAs.  stage_base / block_base count stages and blocks issued by this CTA so far.
    if (warp == 0) {
        // ---- producer: operand tiles and, per stage, the blocks' scales for this tile's rows and columns
        if (lane == 0) {
            uint32_t g = 0;   // global stage counter
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
                for (int it = 0; it < iters; ++it, ++g) {
                    const int s = g % STAGES, ss = g % SST;
                    if (!mbar_wait(empty + s, ((g / STAGES) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(full + s, C::STAGE_BYTES);
                    tma_load_2d(sA + s * C::A_BYTES, &tmA, full + s, it * BK, m0);   // x counts codes
                    tma_load_2d(sB + s * C::B_BYTES, &tmB, full + s, it * BK, n0);
                    if (!mbar_wait(sempty + ss, ((g / SST) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    mbar_arrive_expect_tx(sfull + ss, C::SC_BYTES);
                    float* slot = sSc + ss * C::SC_FLOATS;
                    tma_load_2d(slot, &tmDX, sfull + ss, m0, it * BPS);
                    tma_load_2d(slot + BPS * BM, &tmDW, sfull + ss, n0, it * BPS);
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer: per Q8_0 block two K=16 kind::f16 instructions into that block's own TMEM buffer
        if (lane == 0) {
            uint32_t stage_base = 0, block_base = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
                for (int b = 0; b < nblk; ++b) {
                    const int j = b % BPS;
                    const uint32_t g = stage_base + b / BPS, gb = block_base + b;
                    const int s = g % STAGES, buf = gb % NBUF;
                    if (j == 0) {
                        if (!mbar_wait(full + s, (g / STAGES) & 1, abort_flag, p.err)) { ok = false; break; }
                        tc_fence_after();
                    }
                    if (!mbar_wait(tempty + buf, ((gb / NBUF) & 1) ^ 1, abort_flag, p.err)) { ok = false; break; }
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < 2; ++kk) {   // 16 codes = 32 bytes per instruction
                        const uint64_t ad = smem_desc_sw128(smem_u32(sA + s * C::A_BYTES + j * 64 + kk * 32));
                        const uint64_t bd = smem_desc_sw128(smem_u32(sB + s * C::B_BYTES + j * 64 + kk * 32));
                        mma_f16(tmem + static_cast<uint32_t>(buf * BN), ad, bd, IDESC, kk);
                    }
                    mma_commit(tfull + buf);
                    if (j == BPS - 1 || b == nblk - 1) mma_commit(empty + s);
                }
                stage_base += iters;
                block_base += nblk;
            }
        }
    } else {
        // ---- epilogue warps: drain each block's exact sums and apply the rescale in the reference's order
        const int e = warp - 2;
        const int quarter = warp & 3;
        const int grp = e >> 2;
        const int row = quarter * 32 + lane;
        const int col0 = grp * CPT;
        const uint32_t tbase = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(col0);
        uint32_t stage_base = 0, block_base = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int m0 = (tile / tiles_n) * BM, n0 = (tile % tiles_n) * BN;
            const int grow = m0 + row;
            const int gcol0 = n0 + col0;
            float acc[CPT];
#pragma unroll
            for (int j = 0; j < CPT; ++j) {
                const int c = gcol0 + j;
                acc[j] = (p.bias != nullptr && c < p.N) ? __ldg(p.bias + c) : 0.0f;
            }
            for (int b = 0; b < nblk; ++b) {
                const int j = b % BPS;
                const uint32_t g = stage_base + b / BPS, gb = block_base + b;
                const int ss = g % SST, buf = gb % NBUF;
                if (j == 0 && !mbar_wait(sfull + ss, (g / SST) & 1, abort_flag, p.err)) { ok = false; break; }
                if (!mbar_wait(tfull + buf, (gb / NBUF) & 1, abort_flag, p.err)) { ok = false; break; }
                tc_fence_after();
                const float* slot = sSc + ss * C::SC_FLOATS;
                const float dxr = slot[j * BM + row];
                const float* dw = slot + BPS * BM + j * BN + col0;
                // one 32-column chunk in registers at a time; the TMEM buffer is released after its last load
#pragma unroll
                for (int c = 0; c < CPT / 32; ++c) {
                    uint32_t sv[32];
                    tmem_ld32(tbase + static_cast<uint32_t>(buf * BN + c * 32), sv);
                    tmem_ld_wait();
                    if (c == CPT / 32 - 1) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(tempty + buf);
                    }
                    rescale32(acc + c * 32, sv, dw + c * 32, dxr);
                }
                if (j == BPS - 1 || b == nblk - 1) {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(sempty + ss);
                }
            }
            stage_base += iters;
            block_base += nblk;
            if (!ok) break;
            // Outputs leave through a per-warp 4 KB staging tile and TMA bulk stores: one store moves the warp's
            // 32 rows x 128 B, and the TMA clips rows >= M and columns >= N.
            uint8_t* stage = sOut + e * C::STAGE_OUT_BYTES;
            if constexpr (EPI == EPI_STORE || EPI == EPI_RESID) {
#pragma unroll
                for (int c = 0; c < CPT / 32; ++c) {
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
                    // 128-byte swizzle: 16-byte chunk q of row r sits at chunk q ^ (r mod 8)
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        *reinterpret_cast<float4*>(stage + lane * 128 + ((q ^ (lane & 7)) << 4)) =
                            make_float4(acc[c * 32 + 4 * q], acc[c * 32 + 4 * q + 1], acc[c * 32 + 4 * q + 2], acc[c * 32 + 4 * q + 3]);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if constexpr (EPI == EPI_RESID) tma_reduce_add_2d(&tmOut, gcol0 + c * 32, m0 + quarter * 32, stage);
                        else tma_store_2d(&tmOut, gcol0 + c * 32, m0 + quarter * 32, stage);
                        bulk_commit();
                    }
                }
            } else if constexpr (EPI == EPI_GEGLU_Q8 || EPI == EPI_SWIGLU_Q8 || EPI == EPI_RELU_Q8) {
                // 32 activations per thread and group -> one Q8_0 block of the next product's input:
                // GeGLU groups of 64 columns are [32 GELU inputs | their 32 gates] (ModernBertEncoder.GeGlu,
                // ModernBertEncoder.cs:204-214); ReLU groups are 32 columns (DecisionModel.cs:300).
                // SwiGLU groups are [32 gates | their 32 ups] (DecoderKernels.SiluMultiply, DecoderKernels.cs:97-107).
                constexpr int GW = EPI == EPI_RELU_Q8 ? 32 : 64;
#pragma unroll
                for (int g = 0; g < CPT / GW; ++g) {
                    const int pcol = gcol0 + g * GW;
                    const int blk = pcol / GW;           // output block index (32 codes)
                    float act[32];
                    if constexpr (EPI == EPI_GEGLU_Q8) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) act[j] = __fmul_rn(ref_gelu(acc[g * 64 + j]), acc[g * 64 + 32 + j]);
                    } else if constexpr (EPI == EPI_SWIGLU_Q8) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) act[j] = __fmul_rn(ref_silu(acc[g * 64 + j]), acc[g * 64 + 32 + j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) act[j] = fmaxf(acc[g * 32 + j], 0.0f);
                    }
                    if (lane == 0) bulk_wait_read_all();
                    __syncwarp();
                    float d;
                    quantize_block32_store(act, reinterpret_cast<code_t*>(stage + lane * 64), &d);   // 64 B per row
                    if (pcol < p.N && grow < p.M) p.qsc[static_cast<size_t>(blk) * p.ldqs + grow] = d;
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (pcol < p.N) { tma_store_2d(&tmOut, blk * 32, m0 + quarter * 32, stage); bulk_commit(); }
                    }
                }
            }
        }
        if (lane == 0) bulk_wait_all();
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
    CUtensorMap tA, tB, tDX, tDW, tO;
    int rc = make_tmap_2d(&tA, a.qx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.M, a.K, static_cast<uint64_t>(a.K) * 2, BM, BK);
    if (!rc) rc = make_tmap_2d(&tB, a.qw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.N, a.K, static_cast<uint64_t>(a.K) * 2, BN, BK);
    if (!rc) rc = make_tmap_2d(&tDX, a.dx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.K / 32, a.ldx,
                               static_cast<uint64_t>(a.ldx) * 4, BPS, BM, false);
    if (!rc) rc = make_tmap_2d(&tDW, a.dw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.K / 32, a.ldw,
                               static_cast<uint64_t>(a.ldw) * 4, BPS, BN, false);
    if (!rc) {
        if (EPI == EPI_STORE || EPI == EPI_RESID)
            rc = make_tmap_2d(&tO, a.out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, a.M, a.N, static_cast<uint64_t>(a.ldo) * 4, 32, 32, true);
        else   // codes [M, ldqo] fp16-held, 32 codes (64 B) per row per store, no swizzle
            rc = make_tmap_2d(&tO, a.qout, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, a.M, EPI == EPI_RELU_Q8 ? a.N : a.N / 2,
                              static_cast<uint64_t>(a.ldqo) * 2, 32, 32, false);
    }
    if (rc) return rc;
    auto kern = q8_gemm_kernel<BN, EPI_WARPS, STAGES, EPI>;
    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    static DeviceOnce attr;   // per instantiation
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr.mark(dev);
    }
    KParams p{a.M, a.N, a.K, a.bias, a.out, a.ldo, a.qout, a.ldqo, a.qsc, a.ldqs, a.err};
    int nsm = 0;
    if (int e = sm_count(dev, &nsm)) return e;
    const int tiles = ((a.N + BN - 1) / BN) * ((a.M + BM - 1) / BM);
    const int ctas = tiles < nsm ? tiles : nsm;
    kern<<<ctas, C::THREADS, C::SMEM, stream>>>(tA, tB, tDX, tDW, tO, p);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

int gemm(const GemmArgs& a, cudaStream_t stream) {
    if (a.M <= 0 || a.N <= 0) return OK;
    if (a.K <= 0 || a.K % 32 != 0) { set_error("Q8_0 needs a multiple of 32 inputs"); return ERR_ARGUMENT; }
    if (a.ldx < ((a.M + BM - 1) / BM) * BM || a.ldx % 4) {
        set_error("activation scale stride must cover the rows rounded up to 128 and be a multiple of 4"); return ERR_ARGUMENT;
    }
    if (a.ldw < a.N || a.ldw % 4) { set_error("weight scale stride must cover N and be a multiple of 4"); return ERR_ARGUMENT; }
    if ((reinterpret_cast<uintptr_t>(a.qx) & 15) || (reinterpret_cast<uintptr_t>(a.qw) & 15) ||
        (reinterpret_cast<uintptr_t>(a.dx) & 15) || (reinterpret_cast<uintptr_t>(a.dw) & 15)) {
        set_error("Q8_0 operands and scales must be 16-byte aligned"); return ERR_ARGUMENT;
    }
    if ((a.epi == EPI_STORE || a.epi == EPI_RESID) && ((reinterpret_cast<uintptr_t>(a.out) & 15) || (a.ldo & 3))) {
        set_error("product output must be 16-byte aligned with a row stride that is a multiple of 4"); return ERR_ARGUMENT;
    }
    if ((a.epi == EPI_GEGLU_Q8 || a.epi == EPI_SWIGLU_Q8 || a.epi == EPI_RELU_Q8) &&
        ((reinterpret_cast<uintptr_t>(a.qout) & 15) || (a.ldqo & 7))) {
        set_error("code output must be 16-byte aligned with a row stride that is a multiple of 8"); return ERR_ARGUMENT;
    }
    constexpr int BN = 192, EW = 12, ST = 4;
    switch (a.epi) {
        case EPI_STORE: return launch<BN, EW, ST, EPI_STORE>(a, stream);
        case EPI_RESID: return launch<BN, EW, ST, EPI_RESID>(a, stream);
        case EPI_GEGLU_Q8:
            if (a.N % 64) { set_error("GeGLU product needs whole 64-column groups"); return ERR_ARGUMENT; }
            return launch<BN, EW, ST, EPI_GEGLU_Q8>(a, stream);
        case EPI_SWIGLU_Q8:
            if (a.N % 64) { set_error("SwiGLU product needs whole 64-column groups"); return ERR_ARGUMENT; }
            return launch<BN, EW, ST, EPI_SWIGLU_Q8>(a, stream);
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
                                            code_t* __restrict__ q, float* __restrict__ d, int ldd) {
    const int nb = K / 32;
    const long long gw = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= static_cast<long long>(rows) * nb) return;
    const int r = static_cast<int>(gw / nb), b = static_cast<int>(gw % nb);
    const float v = x[static_cast<size_t>(r) * stride + b * 32 + lane];
    const float amax = warp_max(fabsf(v));
    const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
    q[static_cast<size_t>(r) * K + b * 32 + lane] = __int2half_rn(__float2int_rn(__fmul_rn(v, id)));
    if (lane == 0) d[static_cast<size_t>(b) * ldd + r] = round_fp16(__fdiv_rn(amax, 127.0f));
}

// Q8_0.QuantizeWeightBlock (PackedMatrixQ8_0.cs:20-28): d = amax/127, id = 1/d, q = round half away.
__global__ void quantize_weights_kernel(const float* __restrict__ w, int N, int K, code_t* __restrict__ q,
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
    q[static_cast<size_t>(c) * K + b * 32 + lane] = __int2half_rn(static_cast<int>(roundf(__fmul_rn(v, id))));
    if (lane == 0) d[static_cast<size_t>(b) * ldd + c] = round_fp16(dd);
}

int quantize_activations(const float* x, int rows, int stride, int K, code_t* q, float* d, int ldd,
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

int quantize_weights(const float* w, int N, int K, code_t* q, float* d, int ldd, cudaStream_t stream) {
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

__global__ void widen_codes_kernel(const int8_t* __restrict__ src, code_t* __restrict__ dst, size_t n) {
    const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = __int2half_rn(src[i]);
}

int widen_codes(const int8_t* src, code_t* dst, size_t n, cudaStream_t stream) {
    if (n == 0) return OK;
    widen_codes_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(src, dst, n);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace q8
}  // namespace laya
