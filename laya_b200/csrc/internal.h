// internal.h — host-side declarations shared by the laya_b200 translation units (not part of the C ABI).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include <string>

namespace laya {

// Thread-local error message behind laya_last_error().
void set_error(const std::string& msg);
const char* last_error();

// Status codes (mirrors include/laya_b200.h).
enum Status : int {
    OK = 0,
    ERR_ARGUMENT = 1,
    ERR_OUT_OF_RANGE = 2,
    ERR_NOT_SUPPORTED = 3,
    ERR_CUDA = 4,
    ERR_NOT_FOUND = 5,
    ERR_DEVICE_TIMEOUT = 6,
    ERR_COMM = 7,
};

int cuda_fail(cudaError_t e, const char* what);
#define LAYA_CUDA(call)                                      \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return ::laya::cuda_fail(e_, #call); \
    } while (0)

// Once-per-device launcher set-up (a kernel's dynamic shared-memory limit), safe when several host threads launch at
// once: a race repeats the idempotent set-up call, it never skips it. Devices 64 and above are set up on every call.
struct DeviceOnce {
    std::atomic<uint64_t> bits{0};
    bool done(int dev) const { return dev >= 0 && dev < 64 && ((bits.load(std::memory_order_acquire) >> dev) & 1u); }
    void mark(int dev) {
        if (dev >= 0 && dev < 64) bits.fetch_or(uint64_t{1} << dev, std::memory_order_release);
    }
};

// The device's multiprocessor count, cached per device (thread-safe).
inline int sm_count(int dev, int* out) {
    static std::atomic<int> cache[64];
    if (dev >= 0 && dev < 64) {
        const int v = cache[dev].load(std::memory_order_relaxed);
        if (v > 0) { *out = v; return OK; }
    }
    int v = 0;
    const cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute(MultiProcessorCount)");
    if (dev >= 0 && dev < 64) cache[dev].store(v, std::memory_order_relaxed);
    *out = v;
    return OK;
}

// 2-D tensor map over a row-major [rows, cols] matrix, tile box [box_rows, box_cols]; out-of-range elements read
// as zero.  swizzle128: 128-byte swizzle (MMA operand tiles) or none (plain tiles such as block scales).
int make_tmap_2d(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, uint64_t rows,
                 uint64_t cols, uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_cols, bool swizzle128 = true);

// Launch accounting: every kernel launched by the library bumps this counter (per host thread).
void count_launch(int n = 1);
long long launches();

// ------------------------------------------------------------------------------------------------ Q8_0
namespace q8 {
enum Epi : int {
    EPI_STORE = 0,     // out = acc (fp32)
    EPI_RESID = 1,     // out += acc (fp32 residual stream, in place)
    EPI_GEGLU_Q8 = 2,  // columns come as [32 input | 32 gate] groups: gelu(u)*g, quantized to Q8_0
    EPI_RELU_Q8 = 3,   // relu(acc), quantized to Q8_0
    EPI_SWIGLU_Q8 = 4, // columns come as [32 gate | 32 up] groups: silu(g)*u, quantized to Q8_0
};

// Q8_0 codes live on the device as fp16 values that are exactly the integers -127..127 ("fp16-held codes"), the
// operand form of the kind::f16 tensor-core product; block scales are fp32 (the stored fp16 value, widened).
using code_t = __half;

struct GemmArgs {
    int M, N, K;                 // out[M, N] = X[M, K] · W[N, K]ᵀ (+ bias), K a multiple of 32
    const code_t* qx;            // [M, K] activation codes
    const float* dx; int ldx;    // [K/32, ldx] activation block scales, ldx >= roundup(M, 128), multiple of 4
    const code_t* qw;            // [N, K] weight codes
    const float* dw; int ldw;    // [K/32, ldw] weight block scales, ldw >= N, multiple of 4
    const float* bias;           // [N] or null
    int epi;
    float* out; int ldo;         // EPI_STORE / EPI_RESID
    code_t* qout; int ldqo;      // Q8 epilogues: codes [M, ldqo]
    float* qsc; int ldqs;        // Q8 epilogues: block scales [Nout/32, ldqs]
    int* err;                    // device error word
};
int gemm(const GemmArgs& a, cudaStream_t stream);

// Activation quantizer (Q8_0.QuantizeActivations): x [rows, stride] fp32 -> q [rows, K], d [K/32, ldd].
int quantize_activations(const float* x, int rows, int stride, int K, code_t* q, float* d, int ldd,
                         cudaStream_t stream);
// Weight quantizer (Q8_0.QuantizeWeightBlock over every block): w [N, K] fp32 -> q [N, K], d [K/32, ldd].
int quantize_weights(const float* w, int N, int K, code_t* q, float* d, int ldd, cudaStream_t stream);
// int8 codes -> fp16-held codes (n values).
int widen_codes(const int8_t* src, code_t* dst, size_t n, cudaStream_t stream);
}  // namespace q8

}  // namespace laya
