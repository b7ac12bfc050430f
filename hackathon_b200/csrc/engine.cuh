// The ensemble engine: device weights, the per-symbol state table and the step.
#pragma once
#include <memory>
#include <unordered_map>
#include <vector>

#include "layers.cuh"

namespace b2e {

struct EngineOptions {
  int device = 0;
  int lp = kF32;          // CastLinear storage type of the projection weights
  int capacity = 1;       // state slots (symbols) held on this device
  int max_batch = 1;      // rows per step
  bool graphs = true;     // replay the step from a CUDA graph per batch bucket
  int lanes = 1;          // independent row shares per tower for batches of >= lane_min_rows
  int lane_min_rows = 256;
  int lane_towers = 0xF;  // bit t: tower t takes `lanes` lanes, else one chain over all rows
  bool pdl = false;        // programmatic dependent launch inside each tower's chain
  bool priorities = true;   // the xLSTM tower's chain at high launch priority, the others low
};

class Engine {
 public:
  Engine(const Dims& d, const EngineOptions& o, WeightSource& src);
  ~Engine();

  // Host-buffer step: validates the slots, stages them and the features through
  // pinned memory, enqueues the step, and (wait) copies predictions out.
  void submit(const int* slots, const float* feats, int n);
  void wait(float* preds);
  void step(const int* slots, const float* feats, int n, float* preds) {
    submit(slots, feats, n);
    wait(preds);
  }
  // Device-buffer step on `stream`: slots/features/predictions stay in HBM.
  // Invalid slots zero the live-row count on the device (no row is stepped) and
  // raise the sticky flag read by device_error().
  void step_device(const int* d_slots, const float* d_feats, int n, float* d_preds, cudaStream_t stream);
  int device_error();  // synchronises; returns and clears the flag

  void reset_slots(const int* slots, int n);
  void read_slot(int slot, void* host);
  void write_slot(int slot, const void* host);
  size_t slot_bytes() const { return arena_.slot_bytes(); }
  size_t state_bytes() const { return arena_.bytes(); }
  size_t weight_bytes() const { return pack_.bytes(); }
  int capacity() const { return opt_.capacity; }
  int max_batch() const { return opt_.max_batch; }
  int device() const { return opt_.device; }
  int launches_per_step(int n);  // kernels one step of n rows enqueues
  cudaStream_t stream() const { return s0_; }

 private:
  struct Block {
    std::unique_ptr<Layer> layer;
    size_t o_n1, o_n2, o_f1w, o_f1b, o_f2w, o_f2b;
    const float *n1, *n2;
    const void *f1w, *f1b, *f2w, *f2b;
  };
  struct Tower {
    int kind;
    size_t o_dnw, o_dnb;
    const void *dnw, *dnb;
    std::vector<Block> blocks;
  };
  // One tower over one lane (a contiguous share of the step's rows): its own
  // stream and activations, so the chains of all towers and lanes run concurrently.
  struct Chain {
    uint8_t* scratch = nullptr;  // layer scratch
    float *x = nullptr, *t = nullptr, *tl = nullptr, *u = nullptr;  // tl, u: CastLinear-typed GEMM inputs
    cudaStream_t s = nullptr;
    cudaEvent_t done = nullptr;
  };

  int bucket(int n) const;
  void launch(int n, cudaStream_t s);   // graph replay or eager enqueue
  void enqueue(int rows, cudaStream_t s);
  void tower_forward(const Tower& t, Chain& ch, int idx, const StepCtx& c, const void* up, int ld_up, float* preds);
  int lanes_for(int rows) const;
  void check_host_slots(const int* slots, int n);

  Dims d_;
  EngineOptions opt_;
  WeightPack pack_;
  StateArena arena_;
  std::vector<Tower> towers_;
  std::vector<Chain> chains_;  // [lane][tower]
  int* d_nl_ = nullptr;        // live rows per lane (device)
  // input_up of all four towers as one projection: W [4P][fpad] (features
  // padded with zero columns to a multiple of 8 for the tensor cores), bias
  // [4P], input = the step's features in the CastLinear type [rows][fpad],
  // output [rows][4P] (tower t: columns t*P..)
  int fpad_ = 0;
  size_t o_upw_ = 0, o_upb_ = 0;
  const void *upw_ = nullptr, *upb_ = nullptr;
  void* d_feats_lp_ = nullptr;
  void* d_up_ = nullptr;
  LaunchCfg ln_, ln_bulk_;     // chain kernels / state-streaming kernels
  int prio_hi_ = 0, prio_lo_ = 0;
  size_t o_ow_ = 0, o_ob_ = 0;
  const float *ow_ = nullptr, *ob_ = nullptr;

  // step I/O: [n | pad | slots[max_batch]] [feats max_batch*F] [preds max_batch*4]
  uint8_t* d_io_ = nullptr;
  uint8_t* h_io_ = nullptr;
  int* d_n_ = nullptr;
  int* d_slots_ = nullptr;
  float* d_feats_ = nullptr;
  float* d_preds_ = nullptr;
  int* d_err_ = nullptr;
  size_t feats_off_ = 0, preds_off_ = 0;
  int pending_n_ = -1;

  cudaStream_t s0_ = nullptr;
  cudaEvent_t fork_ = nullptr;
  std::unordered_map<int, cudaGraphExec_t> graphs_;
  std::vector<uint8_t> seen_;  // duplicate-slot check
};

}  // namespace b2e
