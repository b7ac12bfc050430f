// The ensemble engine: device weights, the per-symbol state table and the step.
#pragma once
#include <memory>
#include <unordered_map>
#include <vector>

#include "latency.cuh"
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
  bool pdl = true;         // programmatic dependent launch inside each tower's chain
  bool priorities = true;   // the xLSTM tower's chain at high launch priority, the others low
  bool latency = true;      // host steps of a few rows run as one kernel (latency.cuh)
  // Steps submitted while earlier ones run (submit, submit_device) replay as five
  // graphs - the shared input projection, then one per tower on the tower's own
  // stream - so a tower's chain waits only for the same tower's previous step:
  // the towers of consecutive steps overlap instead of meeting at every step's end.
  bool pipeline = true;
};

class Engine {
 public:
  Engine(const Dims& d, const EngineOptions& o, WeightSource& src);
  ~Engine();

  // Host-buffer step: validates the slots, stages them and the features through
  // pinned memory, enqueues the step, and (wait) copies predictions out. Up to
  // kSets steps may be in flight (wait() returns the oldest): a step's copies
  // run on their own streams, beside the step before it.
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
  // Device-buffer step that does not order its end onto `stream`: the step reads
  // d_slots/d_feats after the work enqueued on `stream` so far and writes
  // d_preds at its end; join_device(stream) makes `stream` wait for every step
  // submitted before it. Between the two, the caller leaves the three buffers
  // alone. Consecutive submits overlap (options.pipeline).
  void submit_device(const int* d_slots, const float* d_feats, int n, float* d_preds, cudaStream_t stream);
  void join_device(cudaStream_t stream);
  int device_error();  // synchronises; returns and clears the flag
  // wait() throws kErrDevice while the flag is set (copied back with each host
  // step's predictions), so a timed-out kernel never passes as an answer.

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
  int latency_rows() const { return lat_ && lat_->ok() ? lat_->max_rows() : 0; }
  int latency_cluster() const { return lat_ && lat_->ok() ? lat_->cluster() : 0; }
  cudaStream_t stream() const { return s0_; }
  static constexpr int kSets = 2;  // step I/O buffer sets

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

  // One step's I/O on the device, [n | lane rows | slots] [feats] [preds], its
  // pinned mirror, and the events that order the set's reuse.
  struct IoSet {
    uint8_t* d_io = nullptr;
    uint8_t* h_io = nullptr;
    int* d_n = nullptr;
    int* d_nl = nullptr;  // live rows per lane
    int* d_slots = nullptr;
    float* d_feats = nullptr;
    float* d_preds = nullptr;
    cudaEvent_t in_ready = nullptr;  // inputs copied in
    cudaEvent_t stepped = nullptr;   // the step's graph finished
    cudaEvent_t done = nullptr;      // predictions copied out: the set is free
    cudaEvent_t head = nullptr;      // the step's input projection finished
    cudaEvent_t tower[4] = {};       // each tower's chain finished (pipelined steps)
    void* d_up = nullptr;            // input_up output of the step [rows][4P], CastLinear type
    void* d_feats_lp = nullptr;      // the features in the CastLinear type [rows][fpad]
    bool used = false;
    int host_n = -1;                 // rows of the host step in flight on this set
  };

  int bucket(int n) const;
  void launch(int n, int b, cudaStream_t s);   // graph replay or eager enqueue, I/O set b
  void enqueue(int rows, int b, cudaStream_t s);
  // pipelined step over set b (inputs in place, ordered on s_head_): the input
  // projection on s_head_, each tower on its chain's stream, joined on s0_
  bool pipelined(int n) const;
  void launch_pipelined(int n, int b);
  void enqueue_head(int rows, int b, cudaStream_t s);
  StepCtx chain_ctx(int t, cudaStream_t s, int rows, const int* n_dev, const int* slots) const;
  template <class F>
  void replay(long long key, cudaStream_t s, F&& enqueue_fn);  // capture once per key, then launch
  void order_after_last_step(cudaStream_t s);  // `s` waits for the last step, wherever it ran
  void drain();
  void tower_forward(const Tower& t, Chain& ch, int idx, const StepCtx& c, const void* up, int ld_up, float* preds);
  int lanes_for(int rows) const;
  void check_host_slots(const int* slots, int n);

  Dims d_;
  EngineOptions opt_;
  WeightPack pack_;
  StateArena arena_;
  std::vector<Tower> towers_;
  std::vector<Chain> chains_;  // [lane][tower]
  // input_up of all four towers as one projection: W [4P][fpad] (features
  // padded with zero columns to a multiple of 8 for the tensor cores), bias
  // [4P], input = the step's features in the CastLinear type [rows][fpad],
  // output [rows][4P] (tower t: columns t*P..)
  int fpad_ = 0;
  size_t o_upw_ = 0, o_upb_ = 0;
  const void *upw_ = nullptr, *upb_ = nullptr;
  LaunchCfg ln_, ln_bulk_;     // chain kernels / state-streaming kernels
  int prio_hi_ = 0, prio_lo_ = 0;
  size_t o_ow_ = 0, o_ob_ = 0;
  const float *ow_ = nullptr, *ob_ = nullptr;

  IoSet io_[kSets];
  size_t slots_off_ = 0, feats_off_ = 0, preds_off_ = 0, err_off_ = 0;  // err: the device error word after the step
  int next_set_ = 0;
  std::vector<int> host_fifo_;  // sets of the host steps in flight, oldest first
  int* d_err_ = nullptr;
  int* d_rs_ = nullptr;         // slots of reset_slots
  int* h_rs_ = nullptr;

  cudaStream_t s0_ = nullptr;     // host steps
  cudaStream_t s_h2d_ = nullptr;  // host steps' input copies
  cudaStream_t s_d2h_ = nullptr;  // host steps' prediction copies
  cudaStream_t s_head_ = nullptr; // pipelined steps' input checks and input projection
  bool last_pipelined_ = false;   // the last step ran pipelined (its towers are ordered by their streams)
  cudaEvent_t fork_ = nullptr;
  cudaEvent_t last_step_ = nullptr;     // recorded after every step
  cudaStream_t last_stream_ = nullptr;  // where it was recorded (null: no step yet)
  std::unordered_map<long long, cudaGraphExec_t> graphs_;  // (bucket, set, segment)
  std::vector<uint8_t> seen_;  // duplicate-slot check
  std::unique_ptr<LatencyPath> lat_;  // one-kernel steps of a few rows
};

}  // namespace b2e
