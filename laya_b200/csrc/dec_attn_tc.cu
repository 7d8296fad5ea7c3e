// dec_attn_tc.cu — the Mica decoder's full attention on the 5th-generation tensor cores (head_dim 128).
//
// Same contract as dec::attention_kernel (decoder_kernels.cu; Qwen35Model.FullAttention, Mica/Models/Qwen35Model.cs:
// 687-731, DecoderKernels.MultiplySigmoid): causal GQA attention of a 64-query tile over the keys of positions
// [0, P + L) of its sequence's cache (P = the sequence's earlier length), softmax in fp32 over fp16 q·k products,
// output · sigmoid(gate) in fp32.  Two query heads of one key/value head share a CTA: their 2 × 64 query rows are the
// M = 128 rows of every MMA, so each K and V tile is loaded once for both.
//   per 64-key tile j (key positions from 0, the same tiles in the same order whatever P is):
//     S = Q·K_jᵀ          tcgen05 kind::f16 (M 128, N 64, K 128) into TMEM columns [0, 64)
//     softmax             one row per thread: causal mask, running max raised only when a tile's max exceeds it by
//                         more than 2^8 (the rescale of O in TMEM is then rare), P in fp16 into TMEM [64, 96)
//     O += P·V_j          A = P from TMEM, B = V_j read N-contiguous (M 128, N 128, K 64) into [128, 256)
// K and V tiles stream through a two-deep cp.async ring; 96 KB of shared memory and 256 TMEM columns let two CTAs
// share an SM, so one CTA's MMA round trips overlap the other's softmax.  A row's arithmetic depends only on its own
// scores and the fixed key tiling, so a read in pieces through a state gives the bits of a read at once (tiles past a
// row are fully masked: no rescale, P = 0, O and the row sum unchanged).
// Every wait on an MMA is bounded (common.cuh).
#include "common.cuh"
#include "decoder.h"
#include "internal.h"

namespace laya {
namespace dat {

constexpr int HD = 128, BQ = 64, BKT = 64, THREADS = 128;
constexpr int Q_SLAB = 128 * 128;                 // 64 dims of 128 rows (bytes)
constexpr int KV_SLAB = BKT * 128;                // 64 dims of 64 rows
constexpr int OFF_Q = 0;                          // [128 rows][128 dims] fp16, two slabs
constexpr int OFF_K = OFF_Q + 2 * Q_SLAB;         // [2 buffers][64 keys][128 dims]
constexpr int OFF_V = OFF_K + 2 * 2 * KV_SLAB;
constexpr int OFF_BAR = OFF_V + 2 * 2 * KV_SLAB;
constexpr int SMEM = 1024 + OFF_BAR + 64;
static_assert(2 * SMEM <= 232448, "two CTAs per SM");
constexpr float LOG2E = 1.4426950408889634f;
constexpr float GAP = 8.0f;                       // log2 units: probabilities stay below 2^8 between rescales

constexpr uint32_t T_S = 0, T_P = 64, T_O = 128;

DEVI uint32_t sw(int r, int ch) { return static_cast<uint32_t>(r * 128 + ((ch ^ (r & 7)) << 4)); }
DEVI void cp16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
DEVI void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
DEVI void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
DEVI uint64_t desc_mn(uint32_t saddr, uint32_t lbo) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}
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
DEVI float ex2(float x) {   // 2^x (ex2.approx; 2^-inf = 0)
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
DEVI uint32_t h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__global__ void __launch_bounds__(THREADS, 2) attention_tc_kernel(dec::AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint64_t* bar_pv = bar_s + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = warp_id();
    const int tile = blockIdx.x, h0 = 2 * blockIdx.y;
    const int kvh = h0 / (a.heads / a.kv_heads);
    const int seq = a.tile_seq[tile], q0 = a.tile_p0[tile];
    const int s0 = a.seq_start[seq], L = a.seq_len[seq], P = a.pos0[seq];
    const int ldq = a.heads * HD, ldkv = a.kv_heads * HD;
    const int ke = P + min(L, q0 + BQ);                 // key positions the tile's last query sees
    const int nk = (ke + BKT - 1) / BKT;
    const __half* kbase = a.kc[seq] + kvh * HD;
    const __half* vbase = a.vc[seq] + kvh * HD;

    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_pv, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) { tmem_alloc(tmem_slot, 256); tmem_relinquish(); }

    // Q: rows 0-63 head h0, 64-127 head h0 + 1, queries q0 .. q0 + 63 (rows past the read zero-filled)
#pragma unroll
    for (int i = 0; i < 128 * 16 / THREADS; ++i) {
        const int e = tid + THREADS * i, r = e >> 4, c = e & 15;
        const int q = q0 + (r & 63), head = h0 + (r >> 6);
        const bool in = q < L;
        cp16(sm + OFF_Q + (c >> 3) * Q_SLAB + sw(r, c & 7),
             a.q16 + static_cast<size_t>(s0 + (in ? q : 0)) * ldq + head * HD + c * 8, in);
    }
    cp_commit();
    auto load_kv = [&](int j) {
        const int b = j & 1;
#pragma unroll
        for (int i = 0; i < BKT * 16 / THREADS; ++i) {
            const int e = tid + THREADS * i, r = e >> 4, c = e & 15;
            const int kp = j * BKT + r;
            const bool in = kp < P + L;
            const size_t off = static_cast<size_t>(in ? kp : 0) * ldkv + c * 8;
            cp16(sm + OFF_K + b * 2 * KV_SLAB + (c >> 3) * KV_SLAB + sw(r, c & 7), kbase + off, in);
            cp16(sm + OFF_V + b * 2 * KV_SLAB + (c >> 3) * KV_SLAB + sw(r, c & 7), vbase + off, in);
        }
        cp_commit();
    };
    load_kv(0);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const uint32_t base = smem_u32(sm);

    constexpr uint32_t ID_S = make_idesc(1, 0, 0, 128, BKT);                  // f16 × f16 → f32, K-major
    constexpr uint32_t ID_PV = make_idesc(1, 0, 0, 128, HD) | (1u << 16);    // A from TMEM, B (V) N-contiguous
    const int row = tid;                                  // this thread's TMEM lane and query row
    const int qi = q0 + (row & 63);
    const bool valid = qi < L;
    const int pq = P + qi;                                // the row's position: keys up to pq are visible
    const float sl2 = a.scale * LOG2E;
    float m_run = -INFINITY, l_run = 0.0f;
    bool ok = true;
    uint32_t ph_s = 0, ph_pv = 0;

    for (int j = 0; j < nk && ok; ++j) {
        // the previous tile's P·V is done before its V buffer is refilled and before P and O are touched
        if (j > 0) {
            ok = __syncthreads_and(mbar_wait(bar_pv, ph_pv, abort_flag, a.err));
            ph_pv ^= 1u;
            if (!ok) break;
        }
        if (j + 1 < nk) { load_kv(j + 1); cp_wait<1>(); } else { cp_wait<0>(); }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();                                  // K_j, V_j (and Q) in shared memory for everyone
        if (tid == 0) {
            tc_fence_after();
            const uint32_t aq = base + OFF_Q, ak = base + OFF_K + (j & 1) * 2 * KV_SLAB;
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk)   // 16 dims per step: slab kk / 4, 32 bytes in
                mma_f16(tmem + T_S, smem_desc_sw128(aq + (kk >> 2) * Q_SLAB + (kk & 3) * 32),
                        smem_desc_sw128(ak + (kk >> 2) * KV_SLAB + (kk & 3) * 32), ID_S, kk > 0 ? 1u : 0u);
            mma_commit(bar_s);
        }
        ok = __syncthreads_and(mbar_wait(bar_s, ph_s, abort_flag, a.err));
        ph_s ^= 1u;
        if (!ok) break;
        tc_fence_after();
        uint32_t sv[64];
        {
            uint32_t x0[32], x1[32];
            tmem_ld32(lane_base + T_S, x0);
            tmem_ld32(lane_base + T_S + 32, x1);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 32; ++c) { sv[c] = x0[c]; sv[32 + c] = x1[c]; }
        }
        float mt = -INFINITY;
#pragma unroll
        for (int c = 0; c < BKT; ++c) {
            const int kp = j * BKT + c;
            const float x = (valid && kp <= pq) ? __uint_as_float(sv[c]) * sl2 : -INFINITY;
            sv[c] = __float_as_uint(x);
            mt = fmaxf(mt, x);
        }
        // raise the running max when the tile's exceeds it by more than GAP (or the row sees its first key)
        const bool raise = mt > m_run + GAP || (m_run == -INFINITY && mt > -INFINITY);
        const float alpha = !raise ? 1.0f : (m_run == -INFINITY ? 0.0f : ex2(m_run - mt));
        // O holds earlier tiles: rescale its row in TMEM.  tcgen05.ld/st are warp-collective, so the whole warp takes
        // the branch when any of its rows raised, the others scaling by exactly 1.
        if (__any_sync(0xffffffffu, raise && j > 0 && m_run > -INFINITY)) {
            const float f = (raise && m_run > -INFINITY) ? alpha : 1.0f;
#pragma unroll
            for (int q = 0; q < HD / 32; ++q) {
                uint32_t o[32];
                tmem_ld32(lane_base + T_O + q * 32, o);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
                st32(lane_base + T_O + q * 32, o);
            }
        }
        if (raise) {
            l_run *= alpha;
            m_run = mt;
        }
        float rs = 0.0f;
        const float mref = m_run == -INFINITY ? 0.0f : m_run;   // a row with nothing visible yet: every p is 0
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            uint32_t ph[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float p0 = ex2(__uint_as_float(sv[32 * q + 2 * e]) - mref);
                const float p1 = ex2(__uint_as_float(sv[32 * q + 2 * e + 1]) - mref);
                rs += p0 + p1;
                ph[e] = h2(p0, p1);
            }
            st16(lane_base + T_P + q * 16, ph);
        }
        l_run += rs;
        st_wait();
        tc_fence_before();
        __syncthreads();                                  // P (and a rescaled O) in TMEM for the issuer
        if (tid == 0) {
            tc_fence_after();
            const uint32_t av = base + OFF_V + (j & 1) * 2 * KV_SLAB;
#pragma unroll
            for (int kk = 0; kk < BKT / 16; ++kk)
                mma_ts(tmem + T_O, tmem + T_P + kk * 8, desc_mn(av + kk * 2048, KV_SLAB), ID_PV, (j > 0 || kk > 0) ? 1u : 0u);
            mma_commit(bar_pv);
        }
    }
    if (ok && nk > 0) ok = __syncthreads_and(mbar_wait(bar_pv, ph_pv, abort_flag, a.err));
    if (ok) {   // CTA-uniform: every thread of every warp takes the TMEM loads; only valid rows store
        tc_fence_after();
        const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
        const size_t t = static_cast<size_t>(s0 + (valid ? qi : 0));
        const int head = h0 + (row >> 6);
        const float* gate = a.qkv + t * a.ld_qkv + head * 2 * HD + HD;
        float* orow = a.out + t * a.ld_out + head * HD;
#pragma unroll 1
        for (int q = 0; q < HD / 32; ++q) {
            uint32_t o[32];
            tmem_ld32(lane_base + T_O + q * 32, o);
            tmem_ld_wait();
            if (!valid) continue;
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
                const int d = 32 * q + e;
                float4 r;
                r.x = __fmul_rn(__uint_as_float(o[e]) * inv, ref_sigmoid(gate[d]));
                r.y = __fmul_rn(__uint_as_float(o[e + 1]) * inv, ref_sigmoid(gate[d + 1]));
                r.z = __fmul_rn(__uint_as_float(o[e + 2]) * inv, ref_sigmoid(gate[d + 2]));
                r.w = __fmul_rn(__uint_as_float(o[e + 3]) * inv, ref_sigmoid(gate[d + 3]));
                *reinterpret_cast<float4*>(orow + d) = r;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

}  // namespace dat

// head_dim 128 with an even number of query heads per key/value head and an error word; ERR_NOT_SUPPORTED otherwise
// (the caller then runs the mma.sync kernel).
int dec_attention_tc(const dec::AttnArgs& a, int n_tiles, int hd, cudaStream_t s) {
    if (hd != dat::HD || !a.err || a.kv_heads <= 0 || a.heads % a.kv_heads || (a.heads / a.kv_heads) % 2)
        return ERR_NOT_SUPPORTED;
    if (n_tiles <= 0) return OK;
    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    static DeviceOnce attr;
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(dat::attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, dat::SMEM));
        attr.mark(dev);
    }
    dat::attention_tc_kernel<<<dim3(n_tiles, a.heads / 2), dat::THREADS, dat::SMEM, s>>>(a);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace laya
