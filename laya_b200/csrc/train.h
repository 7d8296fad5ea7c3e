// train.h — argument blocks of the training-path kernels (internal to the library).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace laya {
namespace bf {
enum Epi : int {
    EPI_BF16 = 0,     // out bf16 = A·Bᵀ (+ bias)
    EPI_F32 = 1,      // out fp32 = A·Bᵀ (+ bias)
    EPI_F32_ADD = 2,  // out fp32 += A·Bᵀ (+ bias), by TMA reduce-add
};
// out[M, N] = A · Bᵀ with A [M, K] and B [N, K] in the logical view; a_mn / b_mn say the operand is stored with the
// M (N) index contiguous instead of K: A as [K, lda] and B as [K, ldb].  Row strides in elements.
struct Args {
    int M, N, K;
    const __nv_bfloat16* A; int lda; int a_mn;
    const __nv_bfloat16* B; int ldb; int b_mn;
    const float* bias;
    int epi;
    void* out; int ldo;
    int* err;
};
int gemm(const Args& a, cudaStream_t stream);
}  // namespace bf
}  // namespace laya
