// common.cuh — sm_100a building blocks shared by the laya_b200 kernels: mbarriers with bounded waits,
// TMA tile loads, tcgen05 (TMEM allocation, MMA issue, commit, TMEM loads) and small numeric helpers.
//
// Every wait on an mbarrier is bounded: after LAYA_WAIT_CYCLES clock cycles without progress the waiting
// thread records LAYA_DEV_ERR_TIMEOUT in the kernel's error word, raises the CTA's abort flag and returns
// false, so a protocol bug ends as an error status on the host instead of a hung GPU.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define DEVI __device__ __forceinline__

#ifndef LAYA_WAIT_CYCLES
#define LAYA_WAIT_CYCLES 4000000000ll   // ~2 s at 2 GHz
#endif

enum : int {
    LAYA_DEV_OK = 0,
    LAYA_DEV_ERR_TIMEOUT = 1,
    LAYA_DEV_ERR_BOUNDS = 2,
};

namespace laya {

DEVI uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

DEVI int warp_id() { return threadIdx.x >> 5; }
DEVI int lane_id() { return threadIdx.x & 31; }

// ------------------------------------------------------------------------------------------------ mbarrier
DEVI void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
DEVI void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
DEVI void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

DEVI void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
DEVI void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// A thread whose phase is not complete is suspended until it completes, or for at most LAYA_WAIT_SUSPEND_NS, so a
// waiting warp takes no issue slots from the warps of its SM sub-partition that have work.
#ifndef LAYA_WAIT_SUSPEND_NS
#define LAYA_WAIT_SUSPEND_NS 20000u
#endif
DEVI bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(LAYA_WAIT_SUSPEND_NS)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false (after recording a timeout in
// *err and raising *abort) if it does not within LAYA_WAIT_CYCLES, or if another role already aborted.
DEVI bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    long long t0 = clock64();
    uint32_t spins = 0;
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((++spins & 63u) == 0) {
            if (*abort) return false;
            if (clock64() - t0 > LAYA_WAIT_CYCLES) {
                atomicExch(err, LAYA_DEV_ERR_TIMEOUT);
                *abort = 1;
                return false;
            }
        }
    }
}

// ------------------------------------------------------------------------------------------------ TMA
DEVI void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2D tiled load into this CTA's own shared memory only, completing on an mbarrier.
DEVI void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Bulk tensor stores from this CTA's shared memory, tracked by bulk groups of the issuing thread.
DEVI void tma_store_2d(const CUtensorMap* map, int x, int y, const void* src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(src))
                 : "memory");
}
// Element-wise fp32 add of the smem tile into global memory (dst += src), performed by the TMA unit.
DEVI void tma_reduce_add_2d(const CUtensorMap* map, int x, int y, const void* src) {
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_u32(src))
                 : "memory");
}
// Untiled bulk copies (16-byte aligned addresses, size a multiple of 16): global → this CTA's shared memory completing
// on an mbarrier, and shared → global tracked by the issuing thread's bulk groups.
DEVI void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
DEVI void bulk_store(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
                 "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
}
DEVI void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
DEVI void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
DEVI void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Warms L2 with a tile a later TMA load will read (no shared-memory write, no completion to wait for).
DEVI void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}

// ------------------------------------------------------------------------------------------------ tcgen05
DEVI void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
DEVI void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
DEVI void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
DEVI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DEVI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] · B[smem]ᵀ, int8 × int8 → int32, one instruction per CTA (single-thread issue).
DEVI void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// bf16/f16 × bf16/f16 → fp32.
DEVI void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on the mbarrier when every tcgen05 op this thread issued so far has completed.
DEVI void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// ------------------------------------------------------------------------------------------------ CTA pairs
// Two CTAs of a cluster (ranks 2k, 2k+1, on the two SMs of one TPC) working one tcgen05 product: the even rank issues
// the M = 256 MMAs, each CTA holds its 128 rows of A, its half of B's N and its 128 accumulator lanes.
DEVI uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Every thread of every CTA of the cluster arrives and waits (release / acquire at cluster scope).
DEVI void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of the same shared-memory offset in cluster CTA `rank`.
DEVI uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
DEVI void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// 2D tiled load into this CTA's own shared memory whose byte count completes on an mbarrier of either CTA of the
// pair (the even rank's, which the MMA issuer waits on).  No multicast: each CTA loads only its own tiles.
DEVI void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t cluster_bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
        : "memory");
}
// One warp of EACH CTA of the pair runs these: the same columns are allocated (freed) in both CTAs' TMEM.
DEVI void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
DEVI void tmem_relinquish_pair() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
DEVI void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A · Bᵀ, M = 256 over the pair; issued by the even rank only.
DEVI void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on the mbarrier at a shared::cluster address (this CTA's or the peer's) when the pair MMAs this
// thread issued so far have completed.
DEVI void mma_commit_pair(uint32_t cluster_bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
                 : "memory");
}

// 32 lanes × 32 consecutive 32-bit columns: thread i of the warp gets row (lane base + i).
DEVI void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
DEVI void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 form): K-major operand, 128-byte swizzle, 8-row atoms of 1024 B.
DEVI uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);      // start address
    d |= static_cast<uint64_t>(1u) << 16;                      // leading byte offset (unused for SW128 K-major)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;              // stride byte offset: 8 rows × 128 B
    d |= static_cast<uint64_t>(1u) << 46;                      // descriptor version (sm_100)
    d |= static_cast<uint64_t>(2u) << 61;                      // SWIZZLE_128B
    return d;
}

// Instruction descriptor: dense, D format (0 f16, 1 f32, 2 s32), A/B formats, both K-major, N, M.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t dfmt, uint32_t afmt, uint32_t bfmt, int M, int N) {
    return (dfmt << 4) | (afmt << 7) | (bfmt << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

// ------------------------------------------------------------------------------------------------ packed fp32
// sm_100 two-wide fp32 arithmetic on 64-bit register pairs (lo, hi); each lane is one IEEE op with round-to-nearest,
// identical to the scalar __fmul_rn / __fsub_rn / __fmaf_rn, in half the issue slots.
DEVI uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
DEVI void f2_unpack(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
DEVI uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
DEVI uint64_t f2_mul(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
DEVI uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
DEVI uint64_t f2_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// ------------------------------------------------------------------------------------------------ numerics
// Exact int32 → fp32 for |s| < 2^22: place s in the mantissa of 1.5·2^23 and subtract it back.
DEVI float i2f_exact(int32_t s) { return __fsub_rn(__int_as_float(s + 0x4B400000), 12582912.0f); }

// fp32 → fp16 → fp32 (round to nearest even), what C# (float)(Half)x gives.
DEVI float round_fp16(float x) { return __half2float(__float2half_rn(x)); }

DEVI float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
DEVI float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The reference's vectorised exp (SimdOps.cs:368-390) and erf (SimdOps.cs:329-356), operation for
// operation, so GELU here gives the reference's bits.  Intrinsics with explicit rounding keep nvcc from
// contracting the separate multiplies and adds into fused ones.
DEVI float ref_exp(float value) {
    float x = fminf(fmaxf(value, -87.3f), 88.7f);
    float n = floorf(__fmaf_rn(x, 1.4426950408889634f, 0.5f));
    float r = __fmaf_rn(n, -0.693359375f, x);
    r = __fmaf_rn(n, 2.12194440e-4f, r);
    float p = 1.0f / 720.0f;
    p = __fmaf_rn(p, r, 1.0f / 120.0f);
    p = __fmaf_rn(p, r, 1.0f / 24.0f);
    p = __fmaf_rn(p, r, 1.0f / 6.0f);
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    float scale = __int_as_float((static_cast<int>(n) + 127) << 23);
    return __fmul_rn(p, scale);
}
DEVI float ref_erf(float value) {
    float sign = value < 0.0f ? -1.0f : 1.0f;
    float ax = fabsf(value);
    float t = __fdiv_rn(1.0f, __fadd_rn(1.0f, __fmul_rn(0.5f, ax)));
    float poly = 0.17087277f;
    poly = __fmaf_rn(poly, t, -0.82215223f);
    poly = __fmaf_rn(poly, t, 1.48851587f);
    poly = __fmaf_rn(poly, t, -1.13520398f);
    poly = __fmaf_rn(poly, t, 0.27886807f);
    poly = __fmaf_rn(poly, t, -0.18628806f);
    poly = __fmaf_rn(poly, t, 0.09678418f);
    poly = __fmaf_rn(poly, t, 0.37409196f);
    poly = __fmaf_rn(poly, t, 1.00002368f);
    poly = __fmaf_rn(poly, t, -1.26551223f);
    poly = __fsub_rn(poly, __fmul_rn(ax, ax));
    float y = __fmul_rn(t, ref_exp(poly));
    return __fmul_rn(sign, ax > 6.0f ? 1.0f : __fsub_rn(1.0f, y));
}
// DecoderKernels.Sigmoid / Silu on Vector<float> (DecoderKernels.cs:150-151): 1 / (1 + exp(−x)) with the exp above.
DEVI float ref_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, ref_exp(-x))); }
DEVI float ref_silu(float x) { return __fmul_rn(x, ref_sigmoid(x)); }
// SimdOps.Gelu (SimdOps.cs:305-323): x * 0.5 * (1 + erf(x / √2)).
DEVI float ref_gelu(float x) {
    return __fmul_rn(__fmul_rn(x, 0.5f), __fadd_rn(1.0f, ref_erf(__fmul_rn(x, 0.70710678118654752f))));
}

}  // namespace laya
