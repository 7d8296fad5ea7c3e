// delta_chunk.cu — the Mica DeltaNet layers' gated delta rule in 64-token chunks on the 5th-generation tensor cores
// (key and value head dims 128), for reads that carry no decoder state.
//
// Replaces, for a stateless prefill, the per-token recurrence of DecoderKernels.GatedDeltaRule128
// (Base/Numerics/DecoderKernels.cs:151-259) and Qwen35Model.Recurrence (Mica/Models/Qwen35Model.cs:924-972):
//     per token t:   S ← g_t·S;   u_t = β_t (v_t − Sᵀk_t);   S ← S + k_t u_tᵀ;   o_t = Sᵀq_t
// Over one chunk of tokens 0..n−1 entered with state S₀, with γ_t = g_0⋯g_t and Γ_ts = g_{s+1}⋯g_t (s ≤ t):
//     S_t = γ_t S₀ + Σ_{s≤t} Γ_ts k_s u_sᵀ
//     (I + A) U = diag(β) V − diag(βγ) K S₀,      A_ts = β_t Γ_ts k_t·k_s  (s < t)
//     U = T₂V − W S₀,   T = (I + A)⁻¹,  T₂ = T diag(β),  W = T diag(βγ) K
//     O = diag(γ) Q S₀ + (Γ ∘ QKᵀ)_{s≤t} U,      S_n = γ_{n−1} S₀ + (diag(Γ_{n−1,s}) K)ᵀ U
// which is the recurrence unrolled (u_t of the per-token form is row t of U).  The summation order differs from the
// per-token sweep, so results agree to rounding, not bit for bit; reads through a decoder state (which must give the
// same bits in pieces as at once, Qwen35State) keep the per-token kernel.
//
// One CTA of four warps per (sequence, value head); thread i owns TMEM lane i.  Everything is held transposed so the
// value index runs down the TMEM lanes: Sᵀ (fp32) never leaves tensor memory, and Sᵀ and Uᵀ reach the MMAs as the
// TMEM A operand (bf16 high and low parts).  Every product is fp32-accurate: hi·hi + lo·hi + hi·lo of bf16 parts.
// Per chunk:
//   load     k, q, v rows (fp32) → bf16 hi/lo tiles in shared memory; β, g → γ and Γ_{n−1,s}; K' = diag(Γ_{n−1,s}) K
//   P1       [K; Q]·Kᵀ                                 (M 128 = keys then queries, N 64, K 128)
//   drain    A (fp32, for the solve) from the key rows; Γ ∘ QKᵀ (bf16 hi/lo) from the query rows
//   solve    T = (I + A)⁻¹ by forward substitution, one column per thread; T₁ = T diag(βγ), T₂ = T diag(β)
//   P2, P3   Wᵀ = Kᵀ T₁ᵀ,  Ũᵀ = Vᵀ T₂ᵀ                 (M 128, N 64, K 64)
//   drain    −W (bf16 hi/lo, over the dead V tile); Sᵀ → S₀ᵀ hi/lo in TMEM, Sᵀ ← γ_{n−1} Sᵀ
//   P4, P5   Uᵀ = Ũᵀ + S₀ᵀ(−W)ᵀ,  X = S₀ᵀ Qᵀ            (A from TMEM; M 128, N 64, K 128)
//   drain    Uᵀ → hi/lo in TMEM
//   P6, P7   Oᵀ = Uᵀ (Γ ∘ QKᵀ)ᵀ,  Sᵀ += Uᵀ K'          (A from TMEM; N 64 and 128, K 64)
//   drain    o_t = γ_t X_t + O_t to the output rows
// Every wait is bounded (common.cuh): a protocol fault ends as an error status, never a hung GPU.
#include "common.cuh"
#include "decoder.h"
#include "internal.h"

namespace laya {
namespace dch {

constexpr int CH = 64, DK = 128, DV = 128, THREADS = 128;

// Shared memory (bytes from a 1024-aligned base).  Tiles are bf16, 128-byte swizzled, 64 columns per slab.
constexpr int SLAB128 = 128 * 128;                  // one 64-column slab of 128 rows
constexpr int SLAB64 = 64 * 128;                    // one 64-column slab of 64 rows
constexpr int OFF_KQ = 0;                           // [K; Q] hi, lo: 128 rows × 128, 2 slabs per part
constexpr int KQ_PART = 2 * SLAB128;
constexpr int OFF_KP = OFF_KQ + 2 * KQ_PART;        // K' hi, lo: 64 rows × 128
constexpr int ROW64_PART = 2 * SLAB64;
constexpr int OFF_V = OFF_KP + 2 * ROW64_PART;      // V hi, lo: 64 rows × 128
constexpr int OFF_NW = OFF_V;                       // −W hi, lo: 128 rows (dk) × 64 (t), over V once P3 is done
constexpr int NW_PART = SLAB128;
constexpr int OFF_T = OFF_V + 2 * ROW64_PART;       // T1 hi, T1 lo, T2 hi, T2 lo: 64 rows (s) × 64 (t) each
constexpr int OFF_AQK = OFF_T + 4 * SLAB64;         // Γ∘QKᵀ hi, lo: 64 rows (t) × 64 (s)
constexpr int OFF_AF = OFF_AQK + 2 * SLAB64;        // A, fp32 [64][AF_LD]
constexpr int AF_LD = 68;                           // float4 rows, conflict-free by quarter warps
constexpr int OFF_TF = OFF_AF + CH * AF_LD * 4;     // T = (I + A)⁻¹, fp32 [64][64]
constexpr int OFF_SC = OFF_TF + CH * CH * 4;        // β, g, γ, Γ_{n−1,s}: 64 floats each
// the load phase stages fp32 rows (64 × 512 B) through two buffers that are free then: the T tiles, and A with T
constexpr int STAGE_A = OFF_T, STAGE_B = OFF_AF;
static_assert(4 * SLAB64 >= CH * 512 && OFF_SC - OFF_AF >= CH * 512, "staging buffers");
constexpr int OFF_BAR = OFF_SC + 4 * CH * 4;
constexpr int SMEM = 1024 + OFF_BAR + 64;
static_assert(NW_PART * 2 <= 2 * ROW64_PART, "−W fits over V");
static_assert(SMEM <= 232448, "shared memory budget");

// TMEM columns (fp32 unless packed bf16 pairs)
constexpr uint32_t T_S = 0;        // Sᵀ [lane j = value dim][col i = key dim]
constexpr uint32_t T_S0 = 128;     // S₀ᵀ bf16 hi (64 packed columns), lo at +64
constexpr uint32_t T_U = 256;      // Ũᵀ, then Uᵀ [j][t]
constexpr uint32_t T_UB = 320;     // Uᵀ bf16 hi (32 packed columns), lo at +32
constexpr uint32_t T_O = 384;      // P1's [KKᵀ; QKᵀ], then Oᵀ
constexpr uint32_t T_X = 448;      // Wᵀ, then X = S₀ᵀQᵀ

DEVI uint32_t sw(int r, int ch) { return static_cast<uint32_t>(r * 128 + ((ch ^ (r & 7)) << 4)); }

// MN-major operand, 128-byte swizzle: 64-element atoms lbo bytes apart, 8-row K groups 1024 B apart.
DEVI uint64_t desc_mn(uint32_t saddr, uint32_t lbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}
// D (+)= A[tmem] · B[smem], A: M 128 rows in the lanes, K 16 packed two bf16 per column.
DEVI void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
DEVI void st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
DEVI void st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
DEVI void st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

DEVI uint32_t bf2(float a, float b) {   // a in the low half
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
// hi and lo bf16 pairs of (a, b): hi = bf16(x), lo = bf16(x − hi)
DEVI void split2(float a, float b, uint32_t& hi, uint32_t& lo) {
    hi = bf2(a, b);
    lo = bf2(__fsub_rn(a, __uint_as_float(hi << 16)), __fsub_rn(b, __uint_as_float(hi & 0xFFFF0000u)));
}
// eight values → one 16-byte chunk of each part
DEVI void split8(const float (&x)[8], uint4& hi, uint4& lo) {
    split2(x[0], x[1], hi.x, lo.x);
    split2(x[2], x[3], hi.y, lo.y);
    split2(x[4], x[5], hi.z, lo.z);
    split2(x[6], x[7], hi.w, lo.w);
}

DEVI void cp16(void* dst, const float* src, bool valid) {   // zero-fills when !valid
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
DEVI void cp4(void* dst, const float* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
DEVI void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
DEVI void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

DEVI void tmem_ld64(uint32_t taddr, float (&v)[64]) {
    uint32_t a[32], b[32];
    tmem_ld32(taddr, a);
    tmem_ld32(taddr + 32, b);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 32; ++i) { v[i] = __uint_as_float(a[i]); v[32 + i] = __uint_as_float(b[i]); }
}

__global__ void __launch_bounds__(THREADS, 1) delta_chunk_kernel(dec::DeltaArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* AF = reinterpret_cast<float*>(sm + OFF_AF);
    float* sb = reinterpret_cast<float*>(sm + OFF_SC);   // β
    float* sg = sb + CH;                                  // g
    float* sgam = sg + CH;                                // γ_t
    float* sgc = sgam + CH;                               // Γ_{n−1,s}
    uint64_t* bar = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const uint32_t base = smem_u32(sm);

    const int tid = threadIdx.x, warp = warp_id(), lane = lane_id();
    const int seq = blockIdx.x, h = blockIdx.y;
    const int kh = h / a.ratio;
    const int s0 = a.seq_start[seq], L = a.seq_len[seq];
    const float* conv = a.conv + static_cast<size_t>(s0) * a.cd;
    const int qoff = kh * DK, koff = a.key_dim + kh * DK, voff = 2 * a.key_dim + h * DV;

    if (tid == 0) {
        mbar_init(bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    {   // S = 0
        uint32_t z[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) z[i] = 0u;
#pragma unroll
        for (int c = 0; c < DK / 32; ++c) st32(lane_base + T_S + c * 32, z);
        st_wait();
    }

    constexpr uint32_t ID_KK = make_idesc(1, 1, 1, 128, 64);                                   // A, B K-major
    constexpr uint32_t ID_MN = make_idesc(1, 1, 1, 128, 64) | (1u << 15) | (1u << 16);         // A, B MN-major
    constexpr uint32_t ID_TS_MN = make_idesc(1, 1, 1, 128, 64) | (1u << 16);                   // A TMEM, B MN-major
    constexpr uint32_t ID_TS_K = make_idesc(1, 1, 1, 128, 64);                                 // A TMEM, B K-major
    constexpr uint32_t ID_TS_MN128 = make_idesc(1, 1, 1, 128, 128) | (1u << 16);               // N 128
    // operand addresses are re-derived inside each round through an opaque move, so the compiler does not hoist
    // every descriptor of every round into registers for the whole chunk loop
    auto opaque = [](uint32_t x) {
        uint32_t y;
        asm volatile("mov.b32 %0, %1;" : "=r"(y) : "r"(x));
        return y;
    };
    uint32_t phase = 0;
    bool ok = true;
    // one round of MMAs issued by thread 0, then every thread waits for their completion
    auto mma_round = [&](auto&& issue) -> bool {
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            issue();
            mma_commit(bar);
        }
        const bool done = mbar_wait(bar, phase, abort_flag, a.err);
        phase ^= 1u;
        tc_fence_after();
        return done;
    };

    const int nch = (L + CH - 1) / CH;
        auto stage_part = [&](int part, int stg, int tb, int nb) {
            const int off = part == 0 ? koff : (part == 1 ? qoff : voff);
#pragma unroll
            for (int i = 0; i < CH * 32 / THREADS; ++i) {
                const int e = tid + THREADS * i, r = e >> 5, m = e & 31;
                const bool in = r < nb;
                cp16(sm + stg + r * 512 + m * 16, conv + static_cast<size_t>(tb + (in ? r : 0)) * a.cd + off + 4 * m, in);
            }
            cp_commit();
        };
        // one staged part → bf16 hi/lo tiles (rows 0-63 of KQ for k, with K' = Γ_{n−1,s}·k beside; 64-127 for q; V)
        auto convert_part = [&](int part, int stg) {
#pragma unroll 4
            for (int i = 0; i < CH * 32 / THREADS; ++i) {
                const int e = tid + THREADS * i, r = e >> 5, m = e & 31;
                const float4 x = *reinterpret_cast<const float4*>(sm + stg + r * 512 + m * 16);
                const int col = 4 * m, slab = col >> 6, ch = (col & 63) >> 3, half = (col & 7) ? 8 : 0;
                uint2 hi, lo;
                split2(x.x, x.y, hi.x, lo.x);
                split2(x.z, x.w, hi.y, lo.y);
                if (part == 0) {
                    uint8_t* d = sm + OFF_KQ + slab * SLAB128 + sw(r, ch) + half;
                    *reinterpret_cast<uint2*>(d) = hi;
                    *reinterpret_cast<uint2*>(d + KQ_PART) = lo;
                    const float gc = sgc[r];
                    uint2 khi, klo;
                    split2(__fmul_rn(x.x, gc), __fmul_rn(x.y, gc), khi.x, klo.x);
                    split2(__fmul_rn(x.z, gc), __fmul_rn(x.w, gc), khi.y, klo.y);
                    uint8_t* dk = sm + OFF_KP + slab * SLAB64 + sw(r, ch) + half;
                    *reinterpret_cast<uint2*>(dk) = khi;
                    *reinterpret_cast<uint2*>(dk + ROW64_PART) = klo;
                } else if (part == 1) {
                    uint8_t* d = sm + OFF_KQ + slab * SLAB128 + sw(CH + r, ch) + half;
                    *reinterpret_cast<uint2*>(d) = hi;
                    *reinterpret_cast<uint2*>(d + KQ_PART) = lo;
                } else {
                    uint8_t* d = sm + OFF_V + slab * SLAB64 + sw(r, ch) + half;
                    *reinterpret_cast<uint2*>(d) = hi;
                    *reinterpret_cast<uint2*>(d + ROW64_PART) = lo;
                }
            }
        };
        // chunk cc's k and q rows into the two staging buffers and its β, g into sb, sg (padding rows: β = 0, g = 1,
        // k = q = v = 0 change nothing); both buffers and sb, sg are free once the previous chunk's P2/P3 are done
        auto issue_kq = [&](int cc) {
            const int tb = cc * CH, nb = min(CH, L - tb);
            stage_part(0, STAGE_A, tb, nb);
            stage_part(1, STAGE_B, tb, nb);
            if (tid < CH) {
                if (tid < nb) {
                    const size_t row = static_cast<size_t>(s0 + tb + tid) * a.vh + h;
                    cp4(sb + tid, a.beta + row);
                    cp4(sg + tid, a.decay + row);
                } else {
                    sb[tid] = 0.0f;
                    sg[tid] = 1.0f;
                }
            }
            cp_commit();
            for (int e = tid; e < nb * 4; e += THREADS)   // and warm L2 with its v rows (512 B each)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(conv + static_cast<size_t>(tb + (e >> 2)) * a.cd + voff + 32 * (e & 3)));
        };
    for (int c = 0; c < nch && ok; ++c) {
        const int t0 = c * CH, n = min(CH, L - t0);
        // ---- load: k and q (staged while the previous chunk finished, or just now for the first), β and g; γ and
        // Γ_{n−1,s} by warp scans; k → K and K' tiles; v staged into the freed buffer; q → Q tiles; v → V tiles
        if (c == 0) issue_kq(0);
        cp_wait<0>();
        __syncthreads();
        if (warp < 2) {   // warp 0: γ_t = g_0⋯g_t (prefix products); warp 1: Γ_{n−1,s} = g_{s+1}⋯g_63 (suffix)
            const float g0 = sg[2 * lane], g1 = sg[2 * lane + 1];
            float p = __fmul_rn(g0, g1);
            if (warp == 0) {
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const float y = __shfl_up_sync(0xffffffffu, p, d);
                    if (lane >= d) p = __fmul_rn(y, p);
                }
                float ex = __shfl_up_sync(0xffffffffu, p, 1);
                if (lane == 0) ex = 1.0f;
                sgam[2 * lane] = __fmul_rn(ex, g0);
                sgam[2 * lane + 1] = p;
            } else {
#pragma unroll
                for (int d = 1; d < 32; d <<= 1) {
                    const float y = __shfl_down_sync(0xffffffffu, p, d);
                    if (lane + d < 32) p = __fmul_rn(p, y);
                }
                float ex = __shfl_down_sync(0xffffffffu, p, 1);
                if (lane == 31) ex = 1.0f;
                sgc[2 * lane + 1] = ex;
                sgc[2 * lane] = __fmul_rn(g1, ex);
            }
        }
        __syncthreads();
        convert_part(0, STAGE_A);
        __syncthreads();       // staging A read: refill it with v
        stage_part(2, STAGE_A, t0, n);
        convert_part(1, STAGE_B);
        cp_wait<0>();
        __syncthreads();
        convert_part(2, STAGE_A);

        // ---- P1: [K; Q]·Kᵀ → T_O
        ok = mma_round([&] {
            const uint32_t kq = opaque(base) + OFF_KQ, tm = opaque(tmem);
            for (int pass = 0; pass < 3; ++pass) {
                const uint32_t pa = pass == 1 ? KQ_PART : 0, pb = pass == 2 ? KQ_PART : 0;
#pragma unroll
                for (int kk = 0; kk < DK / 16; ++kk) {
                    const uint32_t o = (kk >> 2) * SLAB128 + (kk & 3) * 32;
                    mma_f16(tm + T_O, smem_desc_sw128(kq + pa + o), smem_desc_sw128(kq + pb + o), ID_KK,
                            (pass | kk) != 0 ? 1u : 0u);
                }
            }
        });
        if (!ok) break;
        // ---- drain P1: key rows → A (fp32); query rows → Γ ∘ QKᵀ (bf16 hi/lo)
        {
            float v[64];
            tmem_ld64(lane_base + T_O, v);
            if (tid < CH) {
                const int t = tid;
                const float bt = sb[t];
                float G = 1.0f;
#pragma unroll
                for (int s = CH - 1; s >= 0; --s) {
                    if (s < CH - 1) G = s < t ? __fmul_rn(G, sg[s + 1]) : 1.0f;   // Γ_ts = Γ_t,s+1 · g_{s+1}
                    v[s] = s < t ? __fmul_rn(__fmul_rn(bt, G), v[s]) : 0.0f;
                }
#pragma unroll
                for (int m = 0; m < CH / 4; ++m)
                    *reinterpret_cast<float4*>(AF + t * AF_LD + 4 * m) = make_float4(v[4 * m], v[4 * m + 1], v[4 * m + 2], v[4 * m + 3]);
            } else {
                const int t = tid - CH;
                float G = 1.0f;
#pragma unroll
                for (int s = CH - 1; s >= 0; --s) {
                    if (s < CH - 1) G = s < t ? __fmul_rn(G, sg[s + 1]) : 1.0f;
                    v[s] = s <= t ? __fmul_rn(G, v[s]) : 0.0f;
                }
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    float x[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) x[e] = v[8 * ch + e];
                    uint4 hi, lo;
                    split8(x, hi, lo);
                    *reinterpret_cast<uint4*>(sm + OFF_AQK + sw(t, ch)) = hi;
                    *reinterpret_cast<uint4*>(sm + OFF_AQK + SLAB64 + sw(t, ch)) = lo;
                }
            }
        }
        __syncthreads();
        // ---- solve (I + A) T = I in four 16-row blocks: block b's rows first take R = Σ_{s<16b} A_ts T_s (all 128
        // threads: column j, eight rows each), then T_tj = δ_tj − R_tj − Σ_{16b≤s<t} A_ts T_sj by forward substitution
        // inside the block (one thread per column).  T₁ = T diag(βγ), T₂ = T diag(β), stored [s = j][t].
        {
            float* TF = reinterpret_cast<float*>(sm + OFF_TF);
            const int j = tid & (CH - 1), hb = tid >> 6;
#pragma unroll 1
            for (int b = 0; b < CH / 16; ++b) {
                if (b > 0) {
                    float R[8];
#pragma unroll
                    for (int r = 0; r < 8; ++r) R[r] = 0.0f;
                    const float* arow = AF + (16 * b + 8 * hb) * AF_LD;
#pragma unroll 2
                    for (int s4 = 0; s4 < 16 * b; s4 += 4) {
                        const float t0v = TF[(s4 + 0) * CH + j], t1v = TF[(s4 + 1) * CH + j];
                        const float t2v = TF[(s4 + 2) * CH + j], t3v = TF[(s4 + 3) * CH + j];
#pragma unroll
                        for (int r = 0; r < 8; ++r) {
                            const float4 av = *reinterpret_cast<const float4*>(arow + r * AF_LD + s4);
                            R[r] = __fmaf_rn(av.x, t0v, R[r]);
                            R[r] = __fmaf_rn(av.y, t1v, R[r]);
                            R[r] = __fmaf_rn(av.z, t2v, R[r]);
                            R[r] = __fmaf_rn(av.w, t3v, R[r]);
                        }
                    }
#pragma unroll
                    for (int r = 0; r < 8; ++r) TF[(16 * b + 8 * hb + r) * CH + j] = R[r];
                }
                __syncthreads();
                if (tid < CH) {   // column-oriented: once x_v is known, every later row of the block takes its term
                    float ab[16][16];   // the block's A, loaded up front so the 16-step chain waits on no load
#pragma unroll
                    for (int u = 1; u < 16; ++u)
#pragma unroll
                        for (int q = 0; q < (u + 3) / 4; ++q) {
                            const float4 av = *reinterpret_cast<const float4*>(AF + (16 * b + u) * AF_LD + 16 * b + 4 * q);
                            ab[u][4 * q] = av.x; ab[u][4 * q + 1] = av.y; ab[u][4 * q + 2] = av.z; ab[u][4 * q + 3] = av.w;
                        }
                    float acc[16];
#pragma unroll
                    for (int u = 0; u < 16; ++u) acc[u] = b > 0 ? TF[(16 * b + u) * CH + j] : 0.0f;
#pragma unroll
                    for (int v = 0; v < 16; ++v) {
                        const float xv = (16 * b + v == j ? 1.0f : 0.0f) - acc[v];
                        TF[(16 * b + v) * CH + j] = xv;
#pragma unroll
                        for (int u = v + 1; u < 16; ++u) acc[u] = __fmaf_rn(ab[u][v], xv, acc[u]);
                    }
                }
                __syncthreads();
            }
            // threads 0-63 write T₁'s row j, threads 64-127 T₂'s
            const float scale = hb == 0 ? __fmul_rn(sb[j], sgam[j]) : sb[j];
            uint8_t* dst = sm + OFF_T + hb * 2 * SLAB64;
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
                float x[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = __fmul_rn(TF[(8 * ch + e) * CH + j], scale);
                uint4 hi, lo;
                split8(x, hi, lo);
                *reinterpret_cast<uint4*>(dst + sw(j, ch)) = hi;
                *reinterpret_cast<uint4*>(dst + SLAB64 + sw(j, ch)) = lo;
            }
        }
        // ---- P2: Wᵀ = Kᵀ T₁ᵀ → T_X;  P3: Ũᵀ = Vᵀ T₂ᵀ → T_U
        ok = mma_round([&] {
            const uint32_t b0 = opaque(base), tm = opaque(tmem);
            const uint32_t kq = b0 + OFF_KQ, vv = b0 + OFF_V, t1 = b0 + OFF_T, t2 = t1 + 2 * SLAB64;
            for (int pass = 0; pass < 3; ++pass) {
                const uint32_t pa = pass == 1 ? 1 : 0, pb = pass == 2 ? 1 : 0;
#pragma unroll
                for (int kk = 0; kk < CH / 16; ++kk) {
                    mma_f16(tm + T_X, desc_mn(kq + pa * KQ_PART + kk * 2048, SLAB128),
                            desc_mn(t1 + pb * SLAB64 + kk * 2048, SLAB64), ID_MN, (pass | kk) != 0 ? 1u : 0u);
                    mma_f16(tm + T_U, desc_mn(vv + pa * ROW64_PART + kk * 2048, SLAB64),
                            desc_mn(t2 + pb * SLAB64 + kk * 2048, SLAB64), ID_MN, (pass | kk) != 0 ? 1u : 0u);
                }
            }
        });
        if (!ok) break;
        if (c + 1 < nch) issue_kq(c + 1);   // the next chunk's rows land while this one finishes
        // ---- drain: −W → shared [dk][t] (over V); Sᵀ → S₀ᵀ hi/lo in TMEM and γ_{n−1}·Sᵀ back
        {
            float v[64];
            tmem_ld64(lane_base + T_X, v);
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
                float x[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) x[e] = -v[8 * ch + e];
                uint4 hi, lo;
                split8(x, hi, lo);
                *reinterpret_cast<uint4*>(sm + OFF_NW + sw(tid, ch)) = hi;
                *reinterpret_cast<uint4*>(sm + OFF_NW + NW_PART + sw(tid, ch)) = lo;
            }
            const float gl = sgam[CH - 1];
#pragma unroll
            for (int q = 0; q < DK / 32; ++q) {
                uint32_t s[32], hi[16], lo[16];
                tmem_ld32(lane_base + T_S + q * 32, s);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 16; ++e) split2(__uint_as_float(s[2 * e]), __uint_as_float(s[2 * e + 1]), hi[e], lo[e]);
                st16(lane_base + T_S0 + q * 16, hi);
                st16(lane_base + T_S0 + 64 + q * 16, lo);
#pragma unroll
                for (int e = 0; e < 32; ++e) s[e] = __float_as_uint(__fmul_rn(__uint_as_float(s[e]), gl));
                st32(lane_base + T_S + q * 32, s);
            }
            st_wait();
        }
        // ---- P4: Uᵀ += S₀ᵀ(−W)ᵀ → T_U;  P5: X = S₀ᵀQᵀ → T_X
        ok = mma_round([&] {
            const uint32_t b0 = opaque(base), tm = opaque(tmem);
            const uint32_t kq = b0 + OFF_KQ, nw = b0 + OFF_NW;
            for (int pass = 0; pass < 3; ++pass) {
                const uint32_t pa = pass == 1 ? 64 : 0, pb = pass == 2 ? 1 : 0;
#pragma unroll
                for (int kk = 0; kk < DK / 16; ++kk) {
                    const uint32_t at = tm + T_S0 + pa + kk * 8;
                    mma_ts(tm + T_U, at, desc_mn(nw + pb * NW_PART + kk * 2048, NW_PART), ID_TS_MN, 1u);
                    mma_ts(tm + T_X, at, smem_desc_sw128(kq + pb * KQ_PART + (kk >> 2) * SLAB128 + CH * 128 + (kk & 3) * 32),
                           ID_TS_K, (pass | kk) != 0 ? 1u : 0u);
                }
            }
        });
        if (!ok) break;
        // ---- drain: Uᵀ → hi/lo in TMEM
        {
#pragma unroll
            for (int q = 0; q < CH / 32; ++q) {
                uint32_t u[32], hi[16], lo[16];
                tmem_ld32(lane_base + T_U + q * 32, u);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 16; ++e) split2(__uint_as_float(u[2 * e]), __uint_as_float(u[2 * e + 1]), hi[e], lo[e]);
                st16(lane_base + T_UB + q * 16, hi);
                st16(lane_base + T_UB + 32 + q * 16, lo);
            }
            st_wait();
        }
        // ---- P6: Oᵀ = Uᵀ(Γ∘QKᵀ)ᵀ → T_O;  P7: Sᵀ += Uᵀ K' → T_S
        ok = mma_round([&] {
            const uint32_t b0 = opaque(base), tm = opaque(tmem);
            const uint32_t kp = b0 + OFF_KP, aqk = b0 + OFF_AQK;
            for (int pass = 0; pass < 3; ++pass) {
                const uint32_t pa = pass == 1 ? 32 : 0, pb = pass == 2 ? 1 : 0;
#pragma unroll
                for (int kk = 0; kk < CH / 16; ++kk) {
                    const uint32_t at = tm + T_UB + pa + kk * 8;
                    mma_ts(tm + T_O, at, smem_desc_sw128(aqk + pb * SLAB64 + kk * 32), ID_TS_K, (pass | kk) != 0 ? 1u : 0u);
                    mma_ts(tm + T_S, at, desc_mn(kp + pb * ROW64_PART + kk * 2048, SLAB64), ID_TS_MN128, 1u);
                }
            }
        });
        if (!ok) break;
        // ---- drain: o_t = γ_t X_t + O_t
        {
            float* out = a.out + static_cast<size_t>(s0 + t0) * a.ld_out + h * DV + tid;
#pragma unroll
            for (int q = 0; q < CH / 32; ++q) {
                uint32_t o[32], x[32];
                tmem_ld32(lane_base + T_O + q * 32, o);
                tmem_ld32(lane_base + T_X + q * 32, x);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    const int t = 32 * q + e;
                    if (t < n) out[static_cast<size_t>(t) * a.ld_out] = __fmaf_rn(sgam[t], __uint_as_float(x[e]), __uint_as_float(o[e]));
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace dch

// The chunked form for stateless reads (a.chunked) at key and value head dims 128; ERR_NOT_SUPPORTED for anything
// else (the caller then runs the per-token kernel).
int dec_delta_rule_chunked(const dec::DeltaArgs& a, int n_seq, cudaStream_t s) {
    if (!a.chunked || a.dk != dch::DK || a.dv != dch::DV || a.rec || a.snap_begin || !a.err) return ERR_NOT_SUPPORTED;
    if (n_seq <= 0) return OK;
    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    static DeviceOnce attr;
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(dch::delta_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dch::SMEM));
        attr.mark(dev);
    }
    dch::delta_chunk_kernel<<<dim3(n_seq, a.vh), dch::THREADS, dch::SMEM, s>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace laya
