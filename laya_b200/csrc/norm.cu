// norm.cu — LayerNorm kernels of the encoder and head, fused with what surrounds them.
//
//   embed_ln   tok_embeddings gather + LayerNorm        (TrainableDecisionModel.cs:254-285, ModernBertEncoder.cs:131-143)
//   ln_q8      LayerNorm (or identity on layer 0) + Q8_0 activation quantizer for the next projection
//              (ModernBertEncoder.cs:159-171, 177-178 + PackedMatrixQ8_0.cs:35-71; DecisionModel.cs:246-260, 284-298)
//   final_ln   final LayerNorm + the question's type embedding (ModernBertEncoder.cs:185, DecisionModel.cs:146-154)
//
// SimdOps.LayerNorm (SimdOps.cs:234-272) reduces with 8 vector lanes; an octet of threads owns one row here
// and thread l accumulates elements l, l+8, l+16, … exactly as lane l of the reference does, then the lanes
// are combined in a fixed order.  The mean, variance and every output element are therefore the same bits
// as the CPU restatement.  HBM traffic per row: read n fp32, write n fp32 or n int8 + n/32 scales.
#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace laya {

// (a0+a4, a1+a5, a2+a6, a3+a7) then pairwise: every lane of the octet ends with the same bits.
DEVI float octet_hsum(float a) {
    float t = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, 4));
    float u = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
    return __fadd_rn(u, __shfl_xor_sync(0xffffffffu, u, 2));
}
DEVI float octet_max(float a) {
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    return fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
}

enum LnMode { LN_Q8 = 0, LN_FINAL = 1, LN_EMBED = 2 };

template <int NPL, int MODE>
__global__ void __launch_bounds__(256) ln_kernel(LnArgs a) {
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    const int row = gt >> 3, l = gt & 7;
    const bool active = row < a.rows;
    const int r = active ? row : a.rows - 1;   // inactive octets shadow the last row so shuffles stay full
    const int n = a.n;
    const float* src;
    if constexpr (MODE == LN_EMBED) {
        int id = a.ids[r];
        if (id < 0 || id >= a.vocab) {
            if (active && l == 0) atomicExch(a.err, LAYA_DEV_ERR_BOUNDS);
            id = 0;
        }
        src = a.table + static_cast<size_t>(id) * n;
    } else {
        src = a.x + static_cast<size_t>(r) * n;
    }
    float v[NPL];
#pragma unroll
    for (int i = 0; i < NPL; ++i) v[i] = src[l + 8 * i];

    if (a.apply_ln) {
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < NPL; ++i) s = __fadd_rn(s, v[i]);
        const float mean = __fdiv_rn(octet_hsum(s), static_cast<float>(n));
        float var = 0.0f;
#pragma unroll
        for (int i = 0; i < NPL; ++i) { const float dd = __fsub_rn(v[i], mean); var = __fmaf_rn(dd, dd, var); }
        var = __fdiv_rn(octet_hsum(var), static_cast<float>(n));
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const int c = l + 8 * i;
            float y = __fmul_rn(__fmul_rn(__fsub_rn(v[i], mean), inv), a.w[c]);
            if (a.b) y = __fadd_rn(y, a.b[c]);
            v[i] = y;
        }
    }

    if (MODE == LN_Q8 && a.q == nullptr) {   // the fp32-accurate path: hi/lo bf16 parts for a split product
        if (!active) return;
#pragma unroll
        for (int i = 0; i < NPL; ++i) {
            const size_t o = static_cast<size_t>(r) * n + l + 8 * i;
            const __nv_bfloat16 h = __float2bfloat16_rn(v[i]);
            a.hi[o] = h;
            a.lo[o] = __float2bfloat16_rn(__fsub_rn(v[i], __bfloat162float(h)));
        }
        return;
    }
    if constexpr (MODE == LN_Q8) {
        // 32-value blocks: thread l holds elements l, l+8, l+16, l+24 of each block.
#pragma unroll
        for (int blk = 0; blk < NPL / 4; ++blk) {
            float m = 0.0f;
#pragma unroll
            for (int t = 0; t < 4; ++t) m = fmaxf(m, fabsf(v[4 * blk + t]));
            const float amax = octet_max(m);
            const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
            if (active) {
                __half* qrow = a.q + static_cast<size_t>(r) * n + blk * 32 + l;
#pragma unroll
                for (int t = 0; t < 4; ++t) qrow[8 * t] = __int2half_rn(__float2int_rn(__fmul_rn(v[4 * blk + t], id)));
                if (l == 0) a.d[static_cast<size_t>(blk) * a.ldd + r] = round_fp16(__fdiv_rn(amax, 127.0f));
            }
        }
    } else {
        if (!active) return;
        float* o = a.out + static_cast<size_t>(r) * n;
        if (MODE == LN_FINAL && a.temb != nullptr) {
            const float* te = a.temb + static_cast<size_t>(a.qtype[a.tok_item[r]]) * n;
#pragma unroll
            for (int i = 0; i < NPL; ++i) o[l + 8 * i] = __fadd_rn(v[i], te[l + 8 * i]);
        } else {
#pragma unroll
            for (int i = 0; i < NPL; ++i) o[l + 8 * i] = v[i];
        }
    }
}

template <int MODE>
static int ln_dispatch(const LnArgs& a, cudaStream_t stream) {
    if (a.rows <= 0) return OK;
    const int threads = 256;
    const unsigned blocks = static_cast<unsigned>((static_cast<long long>(a.rows) * 8 + threads - 1) / threads);
    switch (a.n) {
        case 128: ln_kernel<16, MODE><<<blocks, threads, 0, stream>>>(a); break;
        case 256: ln_kernel<32, MODE><<<blocks, threads, 0, stream>>>(a); break;
        case 512: ln_kernel<64, MODE><<<blocks, threads, 0, stream>>>(a); break;
        case 768: ln_kernel<96, MODE><<<blocks, threads, 0, stream>>>(a); break;
        case 1024: ln_kernel<128, MODE><<<blocks, threads, 0, stream>>>(a); break;
        default: set_error("hidden size not supported by the LayerNorm kernels (128/256/512/768/1024)"); return ERR_NOT_SUPPORTED;
    }
    count_launch();
    LAYA_CUDA(cudaGetLastError());
    return OK;
}

int ln_q8(const LnArgs& a, cudaStream_t s) { return ln_dispatch<LN_Q8>(a, s); }
int ln_final(const LnArgs& a, cudaStream_t s) { return ln_dispatch<LN_FINAL>(a, s); }
int ln_embed(const LnArgs& a, cudaStream_t s) { return ln_dispatch<LN_EMBED>(a, s); }

}  // namespace laya
