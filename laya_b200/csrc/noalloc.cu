// noalloc.cu — the Q8_0 projection for callers that cannot allocate device memory.
//
// laya_q8_0_linear_device keeps its quantized activations in a context's workspace, which laya_ctx_create
// allocates with cudaMalloc.  Some hosts cannot do that: a process whose device memory is handed out by its own
// pool under a fixed budget, or a plugin running inside someone else's process that may not grow the device
// footprint (and whose latency-critical path cannot afford the implicit device synchronisation cudaMalloc and
// cudaFree may cause).  laya_q8_0_linear_noalloc serves them: the caller passes the input, the weight (codes and
// scales) and the output, and the only scratch — the activation codes, their block scales and a status word — lives
// in the file-scope device array below, which every GPU that loads this library holds until the process exits.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/laya_b200.h"
#include "common.cuh"
#include "internal.h"

namespace {

constexpr size_t kScratchBytes = static_cast<size_t>(LAYA_NOALLOC_SCRATCH_BYTES);
constexpr size_t kStatusBytes = 256;   // the status word, padded to keep the code area 256-byte aligned

// [0, 256): status word of the product's bounded waits; then activation codes [rows, K] (fp16-held);
// then their block scales [K/32, rows rounded up to 128].
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_addr[64] = {};   // device address of g_noalloc_scratch, per device ordinal

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace

using namespace laya;

extern "C" int laya_q8_0_linear_noalloc(const float* x, int rows, int input_stride, const uint16_t* weight_codes,
                                        const float* weight_scales, int ldw, int N, int K, const float* bias, float* y,
                                        int output_stride, void* stream) {
    if (rows < 0 || N <= 0 || K <= 0) { set_error("rows must be >= 0 and N, K positive"); return ERR_ARGUMENT; }
    if (K % 32) { set_error("Q8_0 needs a multiple of 32 inputs, got " + std::to_string(K) + "."); return ERR_ARGUMENT; }
    if (input_stride < K) { set_error("input is too small: input_stride < K"); return ERR_ARGUMENT; }
    if (output_stride < N) { set_error("output is too small: output_stride < N"); return ERR_ARGUMENT; }
    if (ldw < N || ldw % 4) { set_error("weight scale stride must cover N and be a multiple of 4"); return ERR_ARGUMENT; }
    if (rows == 0) return OK;
    if (!x || !weight_codes || !weight_scales || !y) { set_error("null input, weight or output"); return ERR_ARGUMENT; }
    if ((reinterpret_cast<uintptr_t>(weight_codes) & 15) || (reinterpret_cast<uintptr_t>(weight_scales) & 15)) {
        set_error("weight codes and scales must be 16-byte aligned"); return ERR_ARGUMENT;
    }
    if ((reinterpret_cast<uintptr_t>(y) & 15) || (output_stride & 3)) {
        set_error("y must be 16-byte aligned with output_stride a multiple of 4"); return ERR_ARGUMENT;
    }
    const size_t ldx = (static_cast<size_t>(rows) + 127) / 128 * 128;
    const size_t code_bytes = align256(static_cast<size_t>(rows) * K * sizeof(q8::code_t));
    const size_t scale_bytes = static_cast<size_t>(K / 32) * ldx * sizeof(float);
    const size_t need = kStatusBytes + code_bytes + scale_bytes;
    if (need > kScratchBytes) {
        set_error("rows x K too large for the no-allocation scratch: needs " + std::to_string(need) + " bytes, the limit is " +
                  std::to_string(kScratchBytes) + " (about rows·K·2 + rows·K/8 bytes)");
        return ERR_ARGUMENT;
    }

    int dev = 0;
    LAYA_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) { set_error("device ordinal above 63"); return ERR_NOT_SUPPORTED; }
    void* base = nullptr;
    {
        // Set-up, once per device, with that device current: host code may not use the array's name as a device
        // address, so ask the runtime where the array lives on this device.
        std::lock_guard<std::mutex> lock(g_mutex);
        if (!g_scratch_addr[dev]) {
            void* p = nullptr;
            LAYA_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            g_scratch_addr[dev] = p;
        }
        base = g_scratch_addr[dev];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* status = static_cast<int*>(base);
    q8::code_t* codes = reinterpret_cast<q8::code_t*>(static_cast<unsigned char*>(base) + kStatusBytes);
    float* scales = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + kStatusBytes + code_bytes);

    // The array keeps whatever the previous call left.  Two things must start at zero: the status word, and the
    // scales of the padded rows [rows, ldx) of each block row, which the product reads with the rest of its 128-row
    // tile (their accumulators are never stored, but an old call's bytes there could be NaN or Inf).
    LAYA_CUDA(cudaMemsetAsync(status, 0, sizeof(int), s));
    if (ldx > static_cast<size_t>(rows))
        LAYA_CUDA(cudaMemset2DAsync(scales + rows, ldx * sizeof(float), 0, (ldx - rows) * sizeof(float), K / 32, s));
    int rc = q8::quantize_activations(x, rows, input_stride, K, codes, scales, static_cast<int>(ldx), s);
    if (rc != OK) return rc;
    q8::GemmArgs a{};
    a.M = rows; a.N = N; a.K = K;
    a.qx = codes; a.dx = scales; a.ldx = static_cast<int>(ldx);
    a.qw = reinterpret_cast<const q8::code_t*>(weight_codes); a.dw = weight_scales; a.ldw = ldw;
    a.bias = bias; a.epi = q8::EPI_STORE; a.out = y; a.ldo = output_stride;
    a.err = status;
    rc = q8::gemm(a, s);
    if (rc != OK) return rc;
    // The product's waits are bounded; one that gives up writes the status word and leaves y incomplete.  The next
    // call clears the word, so read it now: copy it to the host and wait for the stream.
    int h = 0;
    LAYA_CUDA(cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, s));
    LAYA_CUDA(cudaStreamSynchronize(s));
    if (h == LAYA_DEV_ERR_TIMEOUT) { set_error("a device-side wait of the product timed out; y is not valid"); return ERR_DEVICE_TIMEOUT; }
    if (h != 0) { set_error("the product reported device error " + std::to_string(h) + "; y is not valid"); return ERR_CUDA; }
    return OK;
}
