// Projection GEMMs: C[m, n] = epilogue( sum_k A[m, k] * W[n, k] ).
//
// W is an nn.Linear weight ([out, in], row-major) stored in f32 or in the
// CastLinear low type (example_model.py:68-101). Semantics follow CastLinear
// exactly: with a low-precision weight the input is rounded to the low type,
// products accumulate in f32, the bias (stored in the low type) is added, and the
// result is rounded to the low type before it is widened back to f32
// (example_model.py:92-95). Then, in this order: activation, residual add.
//
// Up to kMaxGroups independent problems of the same (M, N, K) run in one launch
// (BlockLinear's diagonal blocks, model/modules.py:52-79).
#pragma once
#include "common.cuh"

namespace b2e {

constexpr int kMaxGroups = 16;

enum Act : int { kActNone = 0, kActRelu = 1 };

struct GemmGroup {
  const void* A = nullptr;     // [M, K], leading dim lda, type a_type
  const void* W = nullptr;     // [N, K], leading dim ldw, type w_type
  const void* bias = nullptr;  // [N], type bias_type, or null
  float* C = nullptr;          // [M, N] f32 output, leading dim ldc, or null
  void* C_lp = nullptr;        // [M, N] low-type copy of the output, or null
  const float* R = nullptr;    // [M, N] residual added last, or null (may alias C)
};

// Row-wise work fused into the tensor-core GEMM's epilogue when one CTA holds
// whole output rows (N <= 256). In order, per row:
//   v = y (+ R)                         y: acc + bias, rounded, activated
//   v = LayerNorm(v) * ln_w             if ln_w  (biased variance, eps ln_eps)
//   v = v + R2                          if R2
//   C = v                               (f32), C_lp as usual
//   T = RMSNorm(v) * norm_w             if norm_w: to T (f32) and/or T_lp (low type)
//   dot_out[m * dot_ld + dot_col] = v . dot_w + dot_b[0]   if dot_w
struct RowEpi {
  const float* ln_w = nullptr;
  float ln_eps = 1e-5f;
  const float* R2 = nullptr;
  int ldr2 = 0;
  const float* norm_w = nullptr;
  float norm_eps = 1.1920928955078125e-07f;
  float* T = nullptr;
  void* T_lp = nullptr;
  int ldt = 0;
  const float* dot_w = nullptr;
  const float* dot_b = nullptr;
  float* dot_out = nullptr;
  int dot_ld = 0, dot_col = 0;
  bool active() const { return ln_w || R2 || norm_w || dot_w; }
};

struct GemmParams {
  GemmGroup g[kMaxGroups];
  int groups = 1;
  int M_max = 0;               // rows the launch is sized for
  const int* M_dev = nullptr;  // live rows (device), or null to use M_max
  int N = 0, K = 0;
  int lda = 0, ldw = 0, ldc = 0, ldc_lp = 0, ldr = 0;
  int a_type = kF32, w_type = kF32, bias_type = kF32;
  int lp = kF32;      // CastLinear low type; kF32 = plain fp32 nn.Linear
  int round_out = 0;  // round the (acc + bias) to `lp` (CastLinear output)
  int act = kActNone;
  int* err = nullptr;  // device error word for bounded-wait timeouts (tensor-core path)
  RowEpi row;          // needs the tensor-core path and N <= 256 (gemm_tc_row_eligible)
  LaunchCfg ln;        // plain launch by default; the engine's chains set PDL and priority
};

// Enqueue on `stream`. Picks, in order: the tcgen05 tensor-core kernel
// (gemm_tc.cu) for dense low-precision problems (A and W both bf16 or both f16,
// more than 16 rows, K and leading dims multiples of 8), the weight-streaming
// kernel for M_max <= 16, and the tiled SIMT kernel otherwise.
void gemm(const GemmParams& p, cudaStream_t stream);

void gemm_tc_init();    // once per device, before any capture (also runs gemm_simt_init)
void gemm_simt_init();  // kernel attributes of the SIMT kernels
bool gemm_tc_eligible(const GemmParams& p);
bool gemm_tc_row_eligible(const GemmParams& p);  // eligible, and N fits one 256-wide tile
void gemm_tc(const GemmParams& p, cudaStream_t stream);

}  // namespace b2e
