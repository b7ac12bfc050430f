// Shared device/host helpers for the B200 ensemble engine (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <string>
#include <stdexcept>
#include <utility>

namespace b2e {

// ---------------------------------------------------------------- errors

// Host-side failure carrying a message; every C-ABI entry point catches it and
// turns it into a status code plus b2e_last_error().
struct Error : std::runtime_error {
  int code;
  Error(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

enum Status : int {
  kOk = 0,
  kErrInvalid = -1,   // bad argument (size, null pointer, unknown name)
  kErrCuda = -2,      // a CUDA runtime call failed
  kErrWeights = -3,   // a weight tensor is missing or has the wrong size
  kErrCapacity = -4,  // slot or batch outside the engine's capacity
  kErrInternal = -5,
  kErrDevice = -6,    // a kernel recorded a code in the engine's device error word
};

#define B2E_CUDA(expr)                                                              \
  do {                                                                              \
    cudaError_t _e = (expr);                                                        \
    if (_e != cudaSuccess)                                                          \
      throw ::b2e::Error(::b2e::kErrCuda, std::string(#expr) + ": " +               \
                                            cudaGetErrorString(_e) + " (" __FILE__  \
                                            ":" + std::to_string(__LINE__) + ")");  \
  } while (0)

#define B2E_CHECK(cond, code, msg)                       \
  do {                                                   \
    if (!(cond)) throw ::b2e::Error((code), (msg));      \
  } while (0)

// Storage type of the projection ("CastLinear") weights and of the activations
// that feed them: the reference's LINEAR_DTYPE (example_model.py:151-157).
enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

inline size_t dtype_size(int t) { return t == kF32 ? 4 : 2; }

// ------------------------------------------------------- device helpers

template <int T>
struct LowP;
template <>
struct LowP<kBF16> {
  using type = __nv_bfloat16;
  __device__ static float load(const void* p, size_t i) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  }
  __device__ static float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
  __device__ static void store(void* p, size_t i, float v) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  }
};
template <>
struct LowP<kF16> {
  using type = __half;
  __device__ static float load(const void* p, size_t i) {
    return __half2float(reinterpret_cast<const __half*>(p)[i]);
  }
  __device__ static float round(float v) { return __half2float(__float2half_rn(v)); }
  __device__ static void store(void* p, size_t i, float v) {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  }
};
template <>
struct LowP<kF32> {
  using type = float;
  __device__ static float load(const void* p, size_t i) { return reinterpret_cast<const float*>(p)[i]; }
  __device__ static float round(float v) { return v; }
  __device__ static void store(void* p, size_t i, float v) { reinterpret_cast<float*>(p)[i] = v; }
};

// Runtime-dispatched versions for kernels that are not templated on the type.
__device__ __forceinline__ float round_to(int t, float v) {
  return t == kBF16 ? LowP<kBF16>::round(v) : (t == kF16 ? LowP<kF16>::round(v) : v);
}
__device__ __forceinline__ void store_as(int t, void* p, size_t i, float v) {
  if (t == kBF16)
    LowP<kBF16>::store(p, i, v);
  else if (t == kF16)
    LowP<kF16>::store(p, i, v);
  else
    LowP<kF32>::store(p, i, v);
}
__device__ __forceinline__ float load_as(int t, const void* p, size_t i) {
  return t == kBF16 ? LowP<kBF16>::load(p, i) : (t == kF16 ? LowP<kF16>::load(p, i) : LowP<kF32>::load(p, i));
}

// Activations, written as the reference's torch ops define them (float32).
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_(float x) { return x * sigmoidf_(x); }
// F.softplus(beta=1, threshold=20)
__device__ __forceinline__ float softplusf_(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
// F.logsigmoid: min(x,0) - log1p(exp(-|x|))
__device__ __forceinline__ float logsigmoidf_(float x) { return fminf(x, 0.0f) - log1pf(expf(-fabsf(x))); }
// exact (erf) GELU
__device__ __forceinline__ float geluf_(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// Number of live rows: a device-side count (set by the step's H2D copy, so one
// captured graph serves every batch size up to its bucket) or a host constant.
__device__ __forceinline__ int live_rows(const int* n_dev, int n_host) { return n_dev ? *n_dev : n_host; }

// Block-wide sum; every thread gets the result. `red` needs 32 floats.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();  // protect `red` from a previous use
  if (lane == 0) red[wid] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
}

// Streaming (evict-first) 128-bit accesses for recurrent state: each element is
// touched once per step, so it should not displace weights and activations in L2.
__device__ __forceinline__ float4 ld_stream(const float4* p) { return __ldcs(p); }
__device__ __forceinline__ void st_stream(float4* p, float4 v) { __stcs(p, v); }

inline int ceil_div(long a, long b) { return int((a + b - 1) / b); }

// ------------------------------------------------------------ launches
// The engine launches the kernels of a tower's chain with programmatic stream
// serialization (PDL): a kernel's grid is launched as soon as every CTA of its
// predecessor has exited, without the predecessor's completion and memory
// flush in between, and then waits in pdl_wait() until those writes are
// visible. No kernel triggers its successor earlier: successors resident ahead
// of time would hold SM slots that the other towers' kernels need. Every kernel
// calls pdl_wait() before its first global read other than weights, and in
// every thread that reads or writes global memory, so a kernel's completion
// also implies its predecessors' (the chain stays transitive). In a kernel
// launched without the attribute it is a no-op.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Prefetches of weights, issued before pdl_wait(): no predecessor writes them,
// so their lines arrive while the predecessor finishes instead of after the
// kernel's first phase. The CTA's threads take one 128-byte line each, all
// inside [v, v + n).
__device__ __forceinline__ void prefetch_l1(const float* v, int n) {
  if (v == nullptr) return;
  for (int i = threadIdx.x * 32; i < n; i += blockDim.x * 32) asm volatile("prefetch.global.L1 [%0];" ::"l"(v + i));
}
__device__ __forceinline__ void prefetch_l2(const float* v, long long n) {
  if (v == nullptr) return;
  for (long long i = threadIdx.x * 32; i < n; i += blockDim.x * 32LL) asm volatile("prefetch.global.L2 [%0];" ::"l"(v + i));
}

// How a kernel is launched: plain (the C-ABI operators on a caller's stream), or
// with PDL and a scheduling priority (the engine's chains: the HBM-streaming
// state kernels run at low priority so that the short latency-bound kernels of
// the other towers get SMs while they stream).
struct LaunchCfg {
  bool pdl = false;
  bool set_prio = false;
  int prio = 0;
  // Grid of the HBM-streaming state kernels (stream.cuh): -1 = the process-wide
  // default (state_kernel_grid), 0 = one persistent CTA per SM, items strided over
  // the CTAs (the ensemble step: its state kernels run beside other work); w > 0
  // = short CTAs of a few consecutive items, about w waves of two CTAs per SM (a
  // state kernel streaming alone).
  int bulk_waves = -1;
};

template <typename... KArgs, typename... Args>
inline void launch_k(const LaunchCfg& L, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (L.pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (L.set_prio) {
    attr[n].id = cudaLaunchAttributePriority;
    attr[n].val.priority = L.prio;
    ++n;
  }
  cfg.attrs = n ? attr : nullptr;
  cfg.numAttrs = n;
  B2E_CUDA(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

}  // namespace b2e
