// The four recurrent layers of the ensemble and the Block/Tower glue kernels.
#pragma once
#include <memory>
#include <string>

#include "gemm.cuh"
#include "runtime.cuh"

namespace b2e {

// Model dimensions; the derived sizes are the ones the reference's constructors
// compute (model/inference_model.py:30-50, model/mamba2.py:10-46,
// model/retnet.py:20-36, model/hawk.py:56-66, model/xlstm.py:339-353).
struct Dims {
  int H = 0, P = 0, depth = 0, heads = 0, F = 0, m_hs = 64, m_bc = 128;
  int mamba_inner() const { return 2 * H; }
  int mamba_heads() const { return 2 * H / m_hs; }
  int mlstm_inner() const { return 2 * H; }
  int mlstm_heads() const { return heads; }
  int mlstm_hs() const { return 2 * H / heads; }
  int slstm_heads() const { return heads / 2; }
  int slstm_bs() const { return H / (heads / 2); }
  int retnet_hs() const { return H / heads; }
  int hawk_bs() const { return H / 4; }
  void validate() const;
};

enum LayerKind : int { kXLSTM = 0, kMamba2 = 1, kRetNet = 2, kHawk = 3 };
struct LatLayer;  // latency.cuh
const char* layer_name(int kind);

// Everything one enqueue of a step needs besides the layer's own buffers.
struct StepCtx {
  cudaStream_t s = nullptr;
  int rows = 0;               // launch size (the bucket); live rows come from n_dev
  const int* n_dev = nullptr;
  const int* slots = nullptr;  // row -> state slot (device)
  int lp = kF32;              // CastLinear storage type; kF32 = the fp32 path
  int* err = nullptr;         // device error word (bounded waits in tensor-core GEMMs)
  LaunchCfg ln;               // launch of every kernel of the chain
  LaunchCfg ln_bulk;          // launch of the HBM-streaming state kernels
};

class Layer {
 public:
  virtual ~Layer() = default;
  // Append this layer's state leaves, in the reference's init_state order.
  virtual void declare_state(StateArena& a) = 0;
  // Look up and pack weights under `prefix` (e.g. "towers.1.blocks.3.layer.").
  virtual void load(WeightSource& src, WeightPack& pack, const std::string& prefix) = 0;
  virtual void resolve(const WeightPack& pack, const StateArena& a) = 0;
  virtual size_t scratch_bytes(int rows) const = 0;
  // out[r] = (residual ? residual[r] : 0) + layer(in[r]) for the live rows; in,
  // out and residual are [rows][H] f32 and out may alias residual. in_lp, when
  // not null, is `in` already rounded to the CastLinear type (what CastLinear
  // feeds its matmul), so the projections can run on the tensor cores.
  // `post`, when not null, is row work for the layer's final projection
  // (fused_rows(c, H) must hold): the engine passes the Block's norm2 there.
  virtual void forward(const StepCtx& c, const float* in, const void* in_lp, float* out, const float* residual,
                       uint8_t* scratch, const RowEpi* post = nullptr) = 0;

  // The layer's packed weights and state leaves for the latency path (latency.cu
  // names each index per layer kind).
  virtual void latency_desc(LatLayer& L) const = 0;

  static std::unique_ptr<Layer> make(int kind, const Dims& d, int lp);
};

// ----- Block / Tower glue (model/inference_model.py:55-95, 117, 142) -----

// out = x * rsqrt(mean(x^2) + eps) * w   (nn.RMSNorm); out (f32) and/or out_lp
// (the same values in the CastLinear type c.lp) may be null.
void rmsnorm_rows(const StepCtx& c, const float* x, const float* w, float eps, int H, float* out, void* out_lp);
// preds[r*ld + col] = dot(x[r], w) + b[0]     (output_proj, fp32 kept)
void output_proj_rows(const StepCtx& c, const float* x, const float* w, const float* b, int H, float* preds,
                      int ld, int col);
// Enqueue one nn.Linear / CastLinear application (see gemm.cuh). A has type
// `at` (f32, or already the weight's low type); C_lp receives a low-type copy;
// `row` is optional row work fused into the tensor-core epilogue.
void linear(const StepCtx& c, const void* A, int at, int lda, const void* W, int wt, const void* bias, int N, int K,
            float* C, int ldc, int act = 0, const float* R = nullptr, int ldr = 0, void* C_lp = nullptr,
            int ldc_lp = 0, const RowEpi* row = nullptr);
// True when this step's projections run on the tensor cores and a 256-wide tile
// holds a whole hidden-size row, so row norms fuse into GEMM epilogues.
bool fused_rows(const StepCtx& c, int H);
// Set *n_dev = n on the stream (tiny kernel; graph-capturable).
void set_rows(int* n_dev, int n, cudaStream_t s);

}  // namespace b2e
