// b2e_linear_static: the CastLinear projection (b2e_linear) for callers that
// cannot allocate device memory, with its scratch in a file-scope device array.
//
// Who needs it: a host that owns every byte of device memory through its own
// pool and forbids raw cudaMalloc (an inference server's arena, a plugin loaded
// into another framework), and code that must not allocate after start-up
// (latency-bound loops, where cudaMalloc/cudaFree synchronise the device).
// b2e_linear asks such a caller for a device error word before it will use the
// tensor cores, and an f32 input with a bf16/fp16 weight runs on the SIMT
// kernel because the tensor cores need the input already rounded to the
// weight's type. Here both live in g_linear_scratch, so the caller passes only
// its inputs and outputs and still gets the tensor-core kernel.
//
// The array is part of this library's device image: every GPU that loads the
// library holds its kScratchBytes until the process exits. All calls share it,
// so calls that overlap on the GPU (two streams, two host threads) race on it.
#include <algorithm>
#include <functional>
#include <mutex>
#include <string>

#include "../../include/b2e.h"
#include "gemm.cuh"

namespace b2e {
int abi_call(const std::function<void()>& f);
}

using namespace b2e;

namespace {

// Layout: [0, 256) three words - the tensor-core kernel's error word (must read
// 0 before the GEMM starts), the code a call made without h_err left pending,
// and the code a call with h_err reports; [256, 256 + kStageBytes) the input
// rounded to the weight's type (fully rewritten by each call that uses it).
constexpr size_t kHeadBytes = 256;
constexpr size_t kStageBytes = size_t(16) << 20;  // 16 MiB
constexpr size_t kScratchBytes = kHeadBytes + kStageBytes;
constexpr long long kMaxStagedElems = kStageBytes / 2;  // m * k of a rounded input
constexpr int kMaxDevices = 64;

}  // namespace

static __device__ __align__(256) uint8_t g_linear_scratch[kScratchBytes];

namespace {

std::mutex g_mu;
void* g_dev_ptr[kMaxDevices] = {};

// Device address of g_linear_scratch on the current device. In host code the
// array's name is only a host-side stand-in; the address comes from the
// runtime, once per device, the first time this device calls in.
uint8_t* scratch_on_current_device() {
  int dev = 0;
  B2E_CUDA(cudaGetDevice(&dev));
  B2E_CHECK(dev >= 0 && dev < kMaxDevices, kErrInvalid, "b2e_linear_static: device ordinal above 63");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_dev_ptr[dev]) {
    void* p = nullptr;
    B2E_CUDA(cudaGetSymbolAddress(&p, g_linear_scratch));
    g_dev_ptr[dev] = p;
  }
  return static_cast<uint8_t*>(g_dev_ptr[dev]);
}

// Start of a call: a code the last call left in the error word (that call had
// no h_err to report it through) moves to the pending word; the error word
// starts this call at 0.
__global__ void k_err_begin(int* w) {
  if (w[0] != 0) w[1] = w[0];
  w[0] = 0;
}

// End of a call with h_err: report this call's code, or else the pending one,
// and clear both.
__global__ void k_err_report(int* w) {
  w[2] = w[0] != 0 ? w[0] : w[1];
  w[0] = 0;
  w[1] = 0;
}

// x (f32, n elements) rounded to nearest-even in the weight's type: the
// x.to(weight.dtype) of CastLinear.forward (example_model.py:92-95).
template <int T>
__global__ void __launch_bounds__(256) k_round_input(const float* __restrict__ x, long long n, void* out) {
  using LT = typename LowP<T>::type;
  LT* o = static_cast<LT*>(out);
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const long long n4 = n >> 2;
    for (long long i = i0; i < n4; i += stride) {
      const float4 v = reinterpret_cast<const float4*>(x)[i];
      LowP<T>::store(o, 4 * i + 0, v.x);
      LowP<T>::store(o, 4 * i + 1, v.y);
      LowP<T>::store(o, 4 * i + 2, v.z);
      LowP<T>::store(o, 4 * i + 3, v.w);
    }
    for (long long i = 4 * n4 + i0; i < n; i += stride) LowP<T>::store(o, i, x[i]);
  } else {
    for (long long i = i0; i < n; i += stride) LowP<T>::store(o, i, x[i]);
  }
}

}  // namespace

extern "C" int b2e_linear_static(const void* x, int32_t x_dtype, int32_t m, int32_t k, const void* w,
                                 int32_t w_dtype, const void* bias, int32_t n, int32_t act, float* y,
                                 int32_t* h_err, void* stream) {
  return abi_call([&] {
    B2E_CHECK(x && w && y, kErrInvalid, "null operand");
    B2E_CHECK(m > 0 && m <= 65535 * 64 && n > 0 && k > 0, kErrInvalid, "bad GEMM sizes");
    B2E_CHECK(w_dtype == kF32 || w_dtype == kBF16 || w_dtype == kF16, kErrInvalid, "unknown weight dtype");
    B2E_CHECK(x_dtype == kF32 || x_dtype == w_dtype, kErrInvalid, "x must be f32 or the weight's dtype");
    B2E_CHECK(act == kActNone || act == kActRelu, kErrInvalid, "unknown activation");
    const bool stage = x_dtype == kF32 && w_dtype != kF32;
    const long long elems = (long long)m * k;
    if (stage && elems > kMaxStagedElems)
      throw Error(kErrInvalid, "b2e_linear_static: an f32 input with a bf16/fp16 weight is rounded into a "
                               "16 MiB static buffer, so m * k must be at most 8388608 (got " +
                                   std::to_string(elems) + "); use b2e_linear for larger inputs");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint8_t* scratch = scratch_on_current_device();
    int* d_err = reinterpret_cast<int*>(scratch);
    k_err_begin<<<1, 1, 0, s>>>(d_err);
    B2E_CUDA(cudaGetLastError());
    const void* a = x;
    int a_type = x_dtype;
    if (stage) {
      void* staged = scratch + kHeadBytes;
      const int blocks = int(std::min<long long>(ceil_div(elems, 4 * 256), 148 * 8));
      if (w_dtype == kBF16)
        k_round_input<kBF16><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), elems, staged);
      else
        k_round_input<kF16><<<blocks, 256, 0, s>>>(static_cast<const float*>(x), elems, staged);
      B2E_CUDA(cudaGetLastError());
      a = staged;
      a_type = w_dtype;
    }
    gemm_tc_init();
    GemmParams p;
    p.g[0].A = a;
    p.g[0].W = w;
    p.g[0].bias = bias;
    p.g[0].C = y;
    p.M_max = m;
    p.N = n;
    p.K = k;
    p.lda = k;
    p.ldw = k;
    p.ldc = n;
    p.a_type = a_type;
    p.w_type = w_dtype;
    p.bias_type = w_dtype;
    p.round_out = w_dtype != kF32;
    p.act = act;
    p.err = d_err;
    gemm(p, s);
    if (h_err) {
      k_err_report<<<1, 1, 0, s>>>(d_err);
      B2E_CUDA(cudaGetLastError());
      B2E_CUDA(cudaMemcpyAsync(h_err, d_err + 2, sizeof(int), cudaMemcpyDeviceToHost, s));
      B2E_CUDA(cudaStreamSynchronize(s));
    }
  });
}
