// The latency path: a whole ensemble step for a few rows as ONE kernel launch.
//
// A step of the graph path is ~30 kernels per tower block; for one request each
// of them is a few microseconds of launch and dependency latency, so a single
// request costs hundreds of microseconds though it moves only the weights once
// and a few MB of state. Here each tower runs on one thread-block cluster (16
// CTAs, or 8 where 16 cannot be co-scheduled) that walks the tower's blocks as
// a fixed sequence of stages. A stage is one full-vector dependency of the
// reference's math (a projection, a per-head state update); everything
// elementwise or per-row between two such points (norms, convs, gates,
// activations, residuals) is recomputed by every CTA in the next stage's
// prologue. A stage's output slice is written into every CTA's shared memory
// of the cluster (distributed shared memory) and a hardware cluster barrier
// ends the stage. While a CTA waits at that barrier, its slice of the next
// stage's weights and recurrent state is already on its way into shared memory
// (cp.async), so HBM latency overlaps the barrier.
//
// The state table, weights and arithmetic are the engine's own (the same
// packed weights, the same slot-indexed state leaves, the same CastLinear
// rounding points), so a slot can be stepped by either path.
#pragma once
#include <string>
#include <vector>

#include "layers.cuh"

namespace b2e {

constexpr int kLatMaxRows = 4;     // rows one latency step can carry
constexpr int kLatMaxFeatures = 128;
constexpr int kLatMaxW = 24;       // weight pointers of one layer
constexpr int kLatMaxS = 10;       // state leaves of one layer

// One recurrent layer's device pointers, filled by Layer::latency_desc. The
// meaning of each index depends on the layer kind (latency.cu names them).
struct LatLayer {
  const void* w[kLatMaxW] = {};
  float* st[kLatMaxS] = {};
  long long ss[kLatMaxS] = {};  // 4-byte words between slots
};

struct LatBlock {
  LatLayer L;
  const float *n1 = nullptr, *n2 = nullptr;  // Block norm1 / norm2 weights (f32)
  const void *f1w = nullptr, *f1b = nullptr, *f2w = nullptr, *f2b = nullptr;  // SimpleMLP
};

struct LatTower {
  int kind = 0;
  const void *upw = nullptr, *upb = nullptr;  // this tower's rows of input_up [P][fpad], [P]
  const void *dnw = nullptr, *dnb = nullptr;  // input_down [H][P], [H]
  const LatBlock* blocks = nullptr;           // [depth] (device)
};

// Everything one latency kernel reads besides the step's rows.
struct LatModel {
  int H, P, F, fpad, depth, lp;
  int rmax;               // rows the shared-memory carve holds (<= kLatMaxRows)
  uint32_t act_bytes[4];  // per tower: activation bytes, then two stage buffers of buf_bytes
  uint32_t buf_bytes[4];
  int heads, m_hs, m_bc;  // ModelConfig heads; Mamba2 head and B/C sizes
  LatTower t[4];
  const float *ow, *ob;   // output_proj (f32)
  int* err;               // the engine's device error word
};

// The step's rows travel as kernel parameters (no host-to-device copy).
struct LatIO {
  int n;
  int slots[kLatMaxRows];
  float feats[kLatMaxRows * kLatMaxFeatures];
  float* preds;  // [n][4], may be pinned host memory
  int* err_out;  // the error word is copied here (may be pinned host memory)
};

class LatencyPath {
 public:
  // Builds the device descriptors; ok() is false when these dims cannot run
  // here (a stage slice would not fit shared memory, or a cluster shape the
  // hardware cannot schedule), and the engine keeps to its graph path.
  LatencyPath(const Dims& d, int lp, const LatTower (&towers)[4], const std::vector<std::vector<LatBlock>>& blocks,
              const float* ow, const float* ob, int* err);
  ~LatencyPath();
  bool ok() const { return ok_; }
  int max_rows() const { return rows_; }
  int cluster() const { return cl_; }
  int clusters_resident() const { return clusters_; }  // clusters of this shape one GPU co-schedules
  size_t smem_bytes() const { return smem_; }
  const std::string& why_not() const { return why_; }
  void launch(const LatIO& io, cudaStream_t s) const;

 private:
  bool ok_ = false;
  int lp_ = 0, rows_ = 0, cl_ = 0, clusters_ = 0;
  size_t smem_ = 0;
  std::string why_;
  LatModel* d_model_ = nullptr;
  LatBlock* d_blocks_ = nullptr;
};

}  // namespace b2e
