// mma_peak.cu — the tensor-core rate this library's kernels are measured against, measured on the device itself.
//
// One CTA per SM; one thread issues `reps` rounds of four back-to-back tcgen05.mma instructions (one 128-byte k-block:
// K 64 for 16-bit operands, K 128 for int8) of shape M 128 × N into one TMEM accumulator, commits, and waits for the
// last one.  Operands are fixed tiles of pseudo-random values in shared memory (or, for the TS form, A in tensor
// memory), so the loop measures the tensor pipe alone: no loads, no epilogue.  Forms:
//   LAYA_MMA_BF16     kind::f16, bf16 × bf16 → fp32, A and B from shared memory
//   LAYA_MMA_F16      kind::f16, fp16 × fp16 → fp32 (the Q8_0 product's operand form)
//   LAYA_MMA_I8       kind::i8, s8 × s8 → s32
//   LAYA_MMA_BF16_TS  kind::f16 bf16 with A read from tensor memory
//   LAYA_MMA_BF16_MN, LAYA_MMA_BF16_TS_MN  the same with B read N-contiguous (the attention P·V form)
// Returns the elapsed time of the whole launch and the mean cycles per MMA instruction seen by the issuing threads.
#include <cuda_runtime.h>

#include <vector>

#include "../../include/laya_b200.h"
#include "common.cuh"
#include "internal.h"

namespace laya {
namespace mp {

DEVI void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
DEVI void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}

DEVI uint64_t desc_mn(uint32_t saddr, uint32_t lbo_bytes) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

// small pseudo-random operand values: bf16/fp16 in ±[0.5, 1), int8 in [-127, 127]
DEVI uint32_t pattern(uint32_t i, int form) {
    uint32_t h = i * 0x9E3779B1u;
    h ^= h >> 15;
    h *= 0x85EBCA77u;
    h ^= h >> 13;
    if (form == LAYA_MMA_I8) return h & 0x7F7F7F7Fu;
    const uint32_t e = form == LAYA_MMA_F16 ? 0x3800u : 0x3F00u;   // exponent of 0.5 (fp16) / 0.5 (bf16)
    const uint32_t m = form == LAYA_MMA_F16 ? 0x03FFu : 0x007Fu;
    const uint32_t lo = e | (h & m) | ((h >> 16) & 0x8000u), hi = e | ((h >> 8) & m) | (h & 0x8000u);
    return lo | (hi << 16);
}

template <int FORM, int N>
__global__ void __launch_bounds__(128, 1) mma_peak_kernel(int reps, unsigned long long* cycles, int* err) {
    constexpr uint32_t ADT = FORM == LAYA_MMA_F16 ? 0u : 1u;
    // kind::i8: D s32 (2), A/B signed 8-bit (1); kind::f16: D f32 (1), A/B bf16 (1) or f16 (0)
    constexpr bool BMN = FORM == LAYA_MMA_BF16_MN || FORM == LAYA_MMA_BF16_TS_MN;   // B read N-contiguous
    constexpr uint32_t IDESC = (FORM == LAYA_MMA_I8 ? make_idesc(2, 1, 1, 128, N) : make_idesc(1, ADT, ADT, 128, N)) |
                               (BMN ? (1u << 16) : 0u);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                 // 128 rows × 128 B
    uint8_t* sB = smem + 128 * 128;     // 256 rows × 128 B
    uint64_t* bar = reinterpret_cast<uint64_t*>(sB + 256 * 128);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = warp_id(), lane = lane_id();
    for (int i = threadIdx.x; i < (128 + 256) * 128 / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(smem)[i] = pattern(i + 977u * blockIdx.x, FORM);
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    fence_proxy_async_smem();
    if (warp == 0) { tmem_alloc(tmem_slot, 512); tmem_relinquish(); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tA = tmem + 256;   // the TS form's A: 128 lanes × 32 columns (four K-16 steps of bf16 pairs)
    constexpr bool TS = FORM == LAYA_MMA_BF16_TS || FORM == LAYA_MMA_BF16_TS_MN;
    if (TS) {
        uint32_t r[8];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int e = 0; e < 8; ++e) r[e] = pattern(threadIdx.x * 32 + c * 8 + e, FORM);
            tmem_st8(tA + (static_cast<uint32_t>(warp * 32) << 16) + c * 8, r);
        }
        asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
        const uint32_t a = smem_u32(sA), b = smem_u32(sB);
        const long long t0 = clock64();
        for (int r = 0; r < reps; ++r) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
                const uint32_t acc = (r > 0 || kk > 0) ? 1u : 0u;
                // B N-contiguous (as V in P·V): N/64 atoms of [64 K-rows × 128 B] 8 KB apart (32 KB at N 256, the
                // size of sB), 16 K-rows of 128 B per step
                const uint64_t bd = BMN ? desc_mn(b + kk * 2048, 8192) : smem_desc_sw128(b + kk * 32);
                if constexpr (FORM == LAYA_MMA_I8)
                    mma_i8(tmem, smem_desc_sw128(a + kk * 32), bd, IDESC, acc);
                else if constexpr (TS)
                    mma_ts(tmem, tA + kk * 8, bd, IDESC, acc);
                else
                    mma_f16(tmem, smem_desc_sw128(a + kk * 32), bd, IDESC, acc);
            }
        }
        mma_commit(bar);
        const bool ok = mbar_wait(bar, 0, abort_flag, err);
        const long long t1 = clock64();
        if (ok) cycles[blockIdx.x] = static_cast<unsigned long long>(t1 - t0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

constexpr int SMEM = 1024 + (128 + 256) * 128 + 64;

template <int FORM, int N>
int launch(int reps, int ctas, unsigned long long* cyc, int* err, cudaStream_t s) {
    static DeviceOnce attr;
    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (!attr.done(dev)) {
        LAYA_CUDA(cudaFuncSetAttribute(mma_peak_kernel<FORM, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        attr.mark(dev);
    }
    mma_peak_kernel<FORM, N><<<ctas, 128, SMEM, s>>>(reps, cyc, err);
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

template <int FORM>
int launch_n(int n, int reps, int ctas, unsigned long long* cyc, int* err, cudaStream_t s) {
    if (n == 64) return launch<FORM, 64>(reps, ctas, cyc, err, s);
    if (n == 128) return launch<FORM, 128>(reps, ctas, cyc, err, s);
    if (n == 256) return launch<FORM, 256>(reps, ctas, cyc, err, s);
    set_error("N must be 64, 128 or 256");
    return ERR_ARGUMENT;
}

}  // namespace mp
}  // namespace laya

using namespace laya;

extern "C" int laya_mma_peak(int form, int n, int reps, double* ms, double* cycles_per_mma) {
    if (!ms || !cycles_per_mma || reps <= 0 || reps > (1 << 24)) { set_error("invalid argument"); return ERR_ARGUMENT; }
    int dev = 0, nsm = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (int e = sm_count(dev, &nsm)) return e;
    unsigned long long* cyc = nullptr;
    int* err = nullptr;
    LAYA_CUDA(cudaMalloc(&cyc, sizeof(unsigned long long) * nsm + sizeof(int)));
    err = reinterpret_cast<int*>(cyc + nsm);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = OK;
    auto run = [&]() -> int {
        LAYA_CUDA(cudaMemset(cyc, 0, sizeof(unsigned long long) * nsm + sizeof(int)));
        LAYA_CUDA(cudaEventCreate(&e0));
        LAYA_CUDA(cudaEventCreate(&e1));
        auto go = [&]() -> int {
            switch (form) {
                case LAYA_MMA_BF16: return mp::launch_n<LAYA_MMA_BF16>(n, reps, nsm, cyc, err, nullptr);
                case LAYA_MMA_F16: return mp::launch_n<LAYA_MMA_F16>(n, reps, nsm, cyc, err, nullptr);
                case LAYA_MMA_I8: return mp::launch_n<LAYA_MMA_I8>(n, reps, nsm, cyc, err, nullptr);
                case LAYA_MMA_BF16_TS: return mp::launch_n<LAYA_MMA_BF16_TS>(n, reps, nsm, cyc, err, nullptr);
                case LAYA_MMA_BF16_MN: return mp::launch_n<LAYA_MMA_BF16_MN>(n, reps, nsm, cyc, err, nullptr);
                case LAYA_MMA_BF16_TS_MN: return mp::launch_n<LAYA_MMA_BF16_TS_MN>(n, reps, nsm, cyc, err, nullptr);
                default: set_error("unknown MMA form"); return ERR_ARGUMENT;
            }
        };
        if (int r = go()) return r;                 // warm-up (clocks up, TMEM allocator touched)
        LAYA_CUDA(cudaEventRecord(e0, nullptr));
        if (int r = go()) return r;
        LAYA_CUDA(cudaEventRecord(e1, nullptr));
        LAYA_CUDA(cudaEventSynchronize(e1));
        float t = 0;
        LAYA_CUDA(cudaEventElapsedTime(&t, e0, e1));
        *ms = t;
        int h_err = 0;
        LAYA_CUDA(cudaMemcpy(&h_err, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (h_err) { set_error("a device-side wait timed out"); return ERR_DEVICE_TIMEOUT; }
        std::vector<unsigned long long> h(nsm);
        LAYA_CUDA(cudaMemcpy(h.data(), cyc, sizeof(unsigned long long) * nsm, cudaMemcpyDeviceToHost));
        double sum = 0;
        for (auto c : h) sum += static_cast<double>(c);
        *cycles_per_mma = sum / nsm / (4.0 * reps);
        return OK;
    };
    rc = run();
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(cyc);
    return rc;
}
