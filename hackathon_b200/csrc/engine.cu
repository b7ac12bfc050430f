// Ensemble engine (see engine.cuh).
//
// One step = MultiTowerModel.forward over the live rows (model/inference_model.py:
// 119-143): the four towers run concurrently on four streams forked from the step
// stream, each a chain of its Blocks (model/inference_model.py:63-68, 85-95),
// then output_proj per tower into its prediction column. A row's state is read
// and written in place at its slot, so there is no blend pass: an idle symbol's
// slot is never touched (the reference folds idle rows back bit for bit,
// example_model.py:907-949). The step is captured once per batch bucket into a
// CUDA graph and replayed; the live row count is read from device memory, so one
// graph serves every batch size up to its bucket.
#include <algorithm>
#include <cstring>

#include "engine.cuh"
#include "gemm.cuh"
#include "stream.cuh"

namespace b2e {

namespace {

// Live rows of each lane: lane l owns rows [l*per, (l+1)*per) of the step.
__global__ void k_split_rows(const int* n_dev, int* n_lane, int lanes, int per) {
  const int l = threadIdx.x;
  if (l < lanes) n_lane[l] = max(0, min(per, *n_dev - l * per));
}

// Features rounded to the CastLinear type (the x.to(weight.dtype) of input_up,
// example_model.py:92-95), rows padded with zeros from F to fpad columns.
template <int T>
__global__ void k_feats_lp(const float* f, int F, void* out, int fpad, const int* n_dev) {
  const long long total = (long long)(*n_dev) * fpad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / fpad;
    const int c = int(i - r * fpad);
    LowP<T>::store(out, size_t(i), c < F ? f[r * F + c] : 0.0f);
  }
}

__global__ void k_validate(const int* slots, int n, int capacity, int* n_dev, int* err) {
  __shared__ int bad;
  if (threadIdx.x == 0) bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    if (slots[i] < 0 || slots[i] >= capacity) bad = 1;
  __syncthreads();
  if (threadIdx.x == 0) {
    *n_dev = bad ? 0 : n;
    if (bad) *err = 1;
  }
}

}  // namespace

Engine::Engine(const Dims& d, const EngineOptions& o, WeightSource& src) : d_(d), opt_(o) {
  d_.validate();
  B2E_CHECK(o.capacity > 0, kErrInvalid, "capacity must be positive");
  B2E_CHECK(o.max_batch > 0 && o.max_batch <= 65535, kErrInvalid, "max_batch must be in 1..65535");
  B2E_CHECK(o.lp == kF32 || o.lp == kBF16 || o.lp == kF16, kErrInvalid, "unknown linear dtype");
  B2E_CUDA(cudaSetDevice(o.device));
  gemm_tc_init();
  stream_init();
  const int H = d.H, P = d.P, F = d.F, lp = o.lp;

  // ---- weights (strict key names of MultiTowerModel.state_dict())
  towers_.resize(4);
  fpad_ = lp == kF32 ? F : (F + 7) & ~7;
  std::vector<const float*> upw(4), upb(4);
  for (int t = 0; t < 4; ++t) {
    Tower& tw = towers_[t];
    tw.kind = t;  // tower order xLSTM, Mamba2, RetNet, Hawk (model/inference_model.py:107-112)
    const std::string tp = "towers." + std::to_string(t) + ".";
    upw[t] = src.get(tp + "input_up.weight", long(P) * F);
    upb[t] = src.get(tp + "input_up.bias", P);
    tw.o_dnw = pack_.add(src.get(tp + "input_down.weight", long(H) * P), size_t(H) * P, lp);
    tw.o_dnb = pack_.add(src.get(tp + "input_down.bias", H), H, lp);
    tw.blocks.resize(d.depth);
    for (int b = 0; b < d.depth; ++b) {
      Block& bl = tw.blocks[b];
      const std::string bp = tp + "blocks." + std::to_string(b) + ".";
      bl.layer = Layer::make(t, d_, lp);
      bl.o_n1 = pack_.add(src.get(bp + "norm1.weight", H), H, kF32);
      bl.layer->load(src, pack_, bp + "layer.");
      bl.o_n2 = pack_.add(src.get(bp + "norm2.weight", H), H, kF32);
      bl.o_f1w = pack_.add(src.get(bp + "mlp.fc1.weight", long(P) * H), size_t(P) * H, lp);
      bl.o_f1b = pack_.add(src.get(bp + "mlp.fc1.bias", P), P, lp);
      bl.o_f2w = pack_.add(src.get(bp + "mlp.fc2.weight", long(H) * P), size_t(H) * P, lp);
      bl.o_f2b = pack_.add(src.get(bp + "mlp.fc2.bias", H), H, lp);
    }
  }
  {
    const int fp = fpad_;
    o_upw_ = pack_.reserve(size_t(4) * P * fp * dtype_size(lp), [=](uint8_t* d) {
      std::vector<float> row(fp, 0.0f);
      for (int t = 0; t < 4; ++t)
        for (int r = 0; r < P; ++r) {
          std::copy(upw[t] + size_t(r) * F, upw[t] + size_t(r + 1) * F, row.begin());
          convert_f32(row.data(), d + (size_t(t) * P + r) * fp * dtype_size(lp), fp, lp);
        }
    });
    o_upb_ = pack_.add_rows({{upb[0], size_t(P)}, {upb[1], size_t(P)}, {upb[2], size_t(P)}, {upb[3], size_t(P)}}, lp);
  }
  o_ow_ = pack_.add(src.get("output_proj.weight", H), H, kF32);  // fp32 kept (example_model.py:106)
  o_ob_ = pack_.add(src.get("output_proj.bias", 1), 1, kF32);
  src.check_all_used();
  pack_.upload();

  // ---- state table, leaves in iter_state_tensors order (example_model.py:160-176)
  for (auto& tw : towers_)
    for (auto& bl : tw.blocks) bl.layer->declare_state(arena_);
  arena_.allocate(o.capacity);

  for (auto& tw : towers_) {
    tw.dnw = pack_.ptr(tw.o_dnw); tw.dnb = pack_.ptr(tw.o_dnb);
    for (auto& bl : tw.blocks) {
      bl.n1 = pack_.ptr<float>(bl.o_n1); bl.n2 = pack_.ptr<float>(bl.o_n2);
      bl.f1w = pack_.ptr(bl.o_f1w); bl.f1b = pack_.ptr(bl.o_f1b);
      bl.f2w = pack_.ptr(bl.o_f2w); bl.f2b = pack_.ptr(bl.o_f2b);
      bl.layer->resolve(pack_, arena_);
    }
  }
  B2E_CHECK(o.lanes >= 1 && o.lanes <= 8, kErrInvalid, "lanes must be in 1..8");
  chains_.resize(size_t(o.lanes) * 4);
  for (size_t ci = 0; ci < chains_.size(); ++ci) {
    Chain& ch = chains_[ci];
    const Tower& tw = towers_[ci % 4];
    // every chain can carry a whole step (a small bucket runs as one lane)
    const size_t R = o.max_batch;
    size_t scratch = 0;
    for (auto& bl : tw.blocks) scratch = std::max(scratch, bl.layer->scratch_bytes(o.max_batch));
    Carver c{nullptr};
    c.take<float>(R * H);
    c.take<float>(R * H);
    c.take<float>(R * H);
    c.take<float>(R * P);
    const size_t glue = (c.off + 255) & ~size_t(255);
    uint8_t* base = nullptr;
    B2E_CUDA(cudaMalloc(&base, glue + scratch + 256));
    Carver g{base};
    ch.x = g.take<float>(R * H);
    ch.t = g.take<float>(R * H);
    ch.tl = g.take<float>(R * H);
    ch.u = g.take<float>(R * P);
    ch.scratch = base + glue;
    B2E_CUDA(cudaStreamCreateWithFlags(&ch.s, cudaStreamNonBlocking));
    B2E_CUDA(cudaEventCreateWithFlags(&ch.done, cudaEventDisableTiming));
  }
  ow_ = pack_.ptr<float>(o_ow_);
  upw_ = pack_.ptr(o_upw_);
  upb_ = pack_.ptr(o_upb_);
  ob_ = pack_.ptr<float>(o_ob_);

  // ---- step I/O: kSets sets, so a host step's copies overlap the step before
  const size_t R = o.max_batch;
  slots_off_ = 256;  // n at 0, lane row counts from 16
  feats_off_ = (slots_off_ + 4 * R + 255) & ~size_t(255);
  preds_off_ = (feats_off_ + 4 * R * F + 255) & ~size_t(255);
  err_off_ = (preds_off_ + 16 * R + 15) & ~size_t(15);
  const size_t io = err_off_ + 128;
  for (IoSet& st : io_) {
    B2E_CUDA(cudaMalloc(&st.d_io, io));
    B2E_CUDA(cudaMallocHost(&st.h_io, io));
    B2E_CUDA(cudaMemset(st.d_io, 0, io));
    st.d_n = reinterpret_cast<int*>(st.d_io);
    st.d_nl = st.d_n + 4;
    st.d_slots = reinterpret_cast<int*>(st.d_io + slots_off_);
    st.d_feats = reinterpret_cast<float*>(st.d_io + feats_off_);
    st.d_preds = reinterpret_cast<float*>(st.d_io + preds_off_);
    B2E_CUDA(cudaEventCreateWithFlags(&st.in_ready, cudaEventDisableTiming));
    B2E_CUDA(cudaEventCreateWithFlags(&st.stepped, cudaEventDisableTiming));
    B2E_CUDA(cudaEventCreateWithFlags(&st.done, cudaEventDisableTiming));
    B2E_CUDA(cudaEventCreateWithFlags(&st.head, cudaEventDisableTiming));
    for (auto& ev : st.tower) B2E_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    // per set: a pipelined step's input projection runs while the step before still reads its own
    B2E_CUDA(cudaMalloc(&st.d_up, size_t(o.max_batch) * 4 * P * dtype_size(lp)));
    if (lp != kF32) B2E_CUDA(cudaMalloc(&st.d_feats_lp, size_t(o.max_batch) * fpad_ * dtype_size(lp)));
  }
  B2E_CUDA(cudaMalloc(&d_err_, 256));
  B2E_CUDA(cudaMemset(d_err_, 0, 256));
  B2E_CUDA(cudaMalloc(&d_rs_, 4 * R));
  B2E_CUDA(cudaMallocHost(&h_rs_, 4 * R));
  B2E_CUDA(cudaStreamCreateWithFlags(&s0_, cudaStreamNonBlocking));
  B2E_CUDA(cudaStreamCreateWithFlags(&s_h2d_, cudaStreamNonBlocking));
  B2E_CUDA(cudaStreamCreateWithFlags(&s_d2h_, cudaStreamNonBlocking));
  B2E_CUDA(cudaStreamCreateWithFlags(&s_head_, cudaStreamNonBlocking));
  B2E_CUDA(cudaEventCreateWithFlags(&fork_, cudaEventDisableTiming));
  B2E_CUDA(cudaEventCreateWithFlags(&last_step_, cudaEventDisableTiming));
  int prio_low = 0, prio_high = 0;
  B2E_CUDA(cudaDeviceGetStreamPriorityRange(&prio_low, &prio_high));
  ln_.pdl = ln_bulk_.pdl = o.pdl;
  ln_bulk_.bulk_waves = 0;  // persistent state kernels: they run beside the other towers' work
  prio_hi_ = prio_high;
  prio_lo_ = prio_low;
  seen_.assign(o.capacity, 0);

  arena_.reset_all(s0_);
  B2E_CUDA(cudaDeviceSynchronize());

  if (o.latency) {
    // the same packed weights and state leaves, described for the latency kernel
    LatTower lt[4];
    std::vector<std::vector<LatBlock>> lb(4);
    for (int t = 0; t < 4; ++t) {
      const Tower& tw = towers_[t];
      lt[t].kind = tw.kind;
      lt[t].upw = static_cast<const uint8_t*>(upw_) + size_t(t) * P * fpad_ * dtype_size(lp);
      lt[t].upb = static_cast<const uint8_t*>(upb_) + size_t(t) * P * dtype_size(lp);
      lt[t].dnw = tw.dnw;
      lt[t].dnb = tw.dnb;
      for (const Block& bl : tw.blocks) {
        LatBlock b;
        bl.layer->latency_desc(b.L);
        b.n1 = bl.n1; b.n2 = bl.n2;
        b.f1w = bl.f1w; b.f1b = bl.f1b; b.f2w = bl.f2w; b.f2b = bl.f2b;
        lb[t].push_back(b);
      }
    }
    lat_ = std::make_unique<LatencyPath>(d_, lp, lt, lb, ow_, ob_, d_err_);
    B2E_CUDA(cudaDeviceSynchronize());
  }
}

Engine::~Engine() {
  cudaSetDevice(opt_.device);
  cudaDeviceSynchronize();
  for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second);
  for (auto& ch : chains_) {
    if (ch.s) cudaStreamDestroy(ch.s);
    if (ch.done) cudaEventDestroy(ch.done);
    if (ch.x) cudaFree(ch.x);
  }
  for (IoSet& st : io_) {
    if (st.d_io) cudaFree(st.d_io);
    if (st.h_io) cudaFreeHost(st.h_io);
    if (st.in_ready) cudaEventDestroy(st.in_ready);
    if (st.stepped) cudaEventDestroy(st.stepped);
    if (st.done) cudaEventDestroy(st.done);
    if (st.head) cudaEventDestroy(st.head);
    for (auto ev : st.tower)
      if (ev) cudaEventDestroy(ev);
    if (st.d_up) cudaFree(st.d_up);
    if (st.d_feats_lp) cudaFree(st.d_feats_lp);
  }
  if (fork_) cudaEventDestroy(fork_);
  if (last_step_) cudaEventDestroy(last_step_);
  if (s0_) cudaStreamDestroy(s0_);
  if (s_h2d_) cudaStreamDestroy(s_h2d_);
  if (s_d2h_) cudaStreamDestroy(s_d2h_);
  if (s_head_) cudaStreamDestroy(s_head_);
  if (d_err_) cudaFree(d_err_);
  if (d_rs_) cudaFree(d_rs_);
  if (h_rs_) cudaFreeHost(h_rs_);
}

int Engine::bucket(int n) const {
  int b = 1;
  while (b < n) b <<= 1;
  return std::min(b, opt_.max_batch);
}

int Engine::lanes_for(int rows) const {
  return (opt_.lanes > 1 && rows >= opt_.lane_min_rows) ? opt_.lanes : 1;
}

void Engine::tower_forward(const Tower& tw, Chain& ch, int idx, const StepCtx& c, const void* up, int ld_up,
                           float* preds) {
  const int H = d_.H, P = d_.P, F = d_.F, lp = opt_.lp;
  const bool low = lp != kF32;
  // GEMM inputs are written in the CastLinear type (the cast CastLinear applies,
  // example_model.py:93-94): u and tl hold bf16/f16 values when `low`.
  float* u32 = low ? nullptr : ch.u;
  void* ulp = low ? static_cast<void*>(ch.u) : nullptr;
  const float eps = 1.1920928955078125e-07f;  // nn.RMSNorm(eps=None) in float32
  // input_down of relu(input_up(features)) (model/inference_model.py:88-90); the
  // four towers' input_up ran as one projection before the fork
  const bool fuse = fused_rows(c, H);
  const size_t nb = tw.blocks.size();
  if (fuse) {
    // every RMSNorm, and output_proj, run inside the epilogue of the projection
    // that produces their input row (one 128x256 tile holds whole rows)
    RowEpi r0;
    r0.norm_w = tw.blocks[0].n1;
    r0.T = ch.t;
    r0.T_lp = ch.tl;
    r0.ldt = H;
    linear(c, up, lp, ld_up, tw.dnw, lp, tw.dnb, H, P, ch.x, H, kActNone, nullptr, 0, nullptr, 0, &r0);
  } else {
    linear(c, up, lp, ld_up, tw.dnw, lp, tw.dnb, H, P, ch.x, H);
  }
  for (size_t bi = 0; bi < nb; ++bi) {
    const Block& bl = tw.blocks[bi];
    // Block.forward: x = layer(norm1(x)) + x; x = x + mlp(norm2(x)) (model/inference_model.py:63-68)
    if (!fuse) rmsnorm_rows(c, ch.x, bl.n1, eps, H, ch.t, low ? ch.tl : nullptr);
    if (fuse) {
      RowEpi r2;
      r2.norm_w = bl.n2;
      r2.T_lp = ch.tl;
      r2.ldt = H;
      bl.layer->forward(c, ch.t, ch.tl, ch.x, ch.x, ch.scratch, &r2);
    } else {
      bl.layer->forward(c, ch.t, low ? ch.tl : nullptr, ch.x, ch.x, ch.scratch);
      rmsnorm_rows(c, ch.x, bl.n2, eps, H, low ? nullptr : ch.t, low ? ch.tl : nullptr);
    }
    linear(c, low ? static_cast<const void*>(ch.tl) : ch.t, lp, H, bl.f1w, lp, bl.f1b, P, H, u32, P, kActRelu,
           nullptr, 0, ulp, P);                                                       // fc1 + ReLU
    if (fuse) {
      RowEpi r3;
      if (bi + 1 < nb) {  // next Block's norm1
        r3.norm_w = tw.blocks[bi + 1].n1;
        r3.T = ch.t;
        r3.T_lp = ch.tl;
        r3.ldt = H;
      } else {  // shared output_proj (model/inference_model.py:142)
        r3.dot_w = ow_;
        r3.dot_b = ob_;
        r3.dot_out = preds;
        r3.dot_ld = 4;
        r3.dot_col = idx;
      }
      linear(c, ch.u, lp, P, bl.f2w, lp, bl.f2b, H, P, ch.x, H, kActNone, ch.x, H, nullptr, 0, &r3);
    } else {
      linear(c, ch.u, lp, P, bl.f2w, lp, bl.f2b, H, P, ch.x, H, kActNone, ch.x, H);  // fc2 + residual
    }
  }
  if (!fuse) output_proj_rows(c, ch.x, ow_, ob_, H, preds, 4, idx);  // shared output_proj (model/inference_model.py:142)
}

void Engine::enqueue_head(int rows, int b, cudaStream_t s) {
  const IoSet& io = io_[b];
  const int L = lanes_for(rows);
  const int per = (rows + L - 1) / L;
  k_split_rows<<<1, 32, 0, s>>>(io.d_n, io.d_nl, L, per);
  B2E_CUDA(cudaGetLastError());
  // input_up of the four towers, one projection over all rows
  const int P = d_.P, F = d_.F, lp = opt_.lp;
  StepCtx c0;
  c0.s = s;
  c0.rows = rows;
  c0.n_dev = io.d_n;
  c0.slots = io.d_slots;
  c0.lp = lp;
  c0.err = d_err_;
  c0.ln = ln_;
  if (lp != kF32) {
    const int blocks = std::max(1, std::min(ceil_div(long(rows) * fpad_, 256 * 4), 148 * 4));
    if (lp == kBF16)
      k_feats_lp<kBF16><<<blocks, 256, 0, s>>>(io.d_feats, F, io.d_feats_lp, fpad_, io.d_n);
    else
      k_feats_lp<kF16><<<blocks, 256, 0, s>>>(io.d_feats, F, io.d_feats_lp, fpad_, io.d_n);
    B2E_CUDA(cudaGetLastError());
    linear(c0, io.d_feats_lp, lp, fpad_, upw_, lp, upb_, 4 * P, fpad_, nullptr, 0, kActRelu, nullptr, 0, io.d_up, 4 * P);
  } else {
    linear(c0, io.d_feats, kF32, F, upw_, kF32, upb_, 4 * P, F, static_cast<float*>(io.d_up), 4 * P, kActRelu);
  }
}

StepCtx Engine::chain_ctx(int t, cudaStream_t s, int rows, const int* n_dev, const int* slots) const {
  StepCtx c;
  c.s = s;
  c.rows = rows;
  c.n_dev = n_dev;
  c.slots = slots;
  c.lp = opt_.lp;
  c.err = d_err_;
  c.ln = ln_;
  c.ln_bulk = ln_bulk_;
  if (opt_.priorities && prio_hi_ != prio_lo_) {
    // the xLSTM and Mamba2 towers' chains are the longest: their kernels
    // take SM slots first
    c.ln.set_prio = c.ln_bulk.set_prio = true;
    c.ln.prio = c.ln_bulk.prio = t <= 1 ? prio_hi_ : prio_lo_;
  }
  return c;
}

void Engine::enqueue(int rows, int b, cudaStream_t s) {
  const IoSet& io = io_[b];
  const int L = lanes_for(rows);
  const int per = (rows + L - 1) / L;
  const int P = d_.P, lp = opt_.lp;
  enqueue_head(rows, b, s);
  B2E_CUDA(cudaEventRecord(fork_, s));
  for (int l = 0; l < L; ++l) {
    for (int t = 0; t < 4; ++t) {
      // a tower outside lane_towers runs as one chain over all rows (lane 0)
      const bool split = L > 1 && ((opt_.lane_towers >> t) & 1);
      if (!split && l > 0) continue;
      Chain& ch = chains_[size_t(l) * 4 + t];
      B2E_CUDA(cudaStreamWaitEvent(ch.s, fork_, 0));
      const StepCtx c = chain_ctx(t, ch.s, split ? per : rows, split ? io.d_nl + l : io.d_n, io.d_slots + size_t(l) * per);
      const void* up = static_cast<const uint8_t*>(io.d_up) + (size_t(l) * per * 4 * P + size_t(t) * P) * dtype_size(lp);
      tower_forward(towers_[t], ch, t, c, up, 4 * P, io.d_preds + size_t(l) * per * 4);
      B2E_CUDA(cudaEventRecord(ch.done, ch.s));
    }
  }
  for (int l = 0; l < L; ++l)
    for (int t = 0; t < 4; ++t)
      if (l == 0 || ((opt_.lane_towers >> t) & 1)) B2E_CUDA(cudaStreamWaitEvent(s, chains_[size_t(l) * 4 + t].done, 0));
}

template <class F>
void Engine::replay(long long key, cudaStream_t s, F&& enqueue_fn) {
  if (!opt_.graphs) {
    enqueue_fn(s);
    return;
  }
  auto it = graphs_.find(key);
  if (it == graphs_.end()) {
    // Capture on a private stream so the caller's stream is never in capture mode.
    cudaGraph_t g = nullptr;
    B2E_CUDA(cudaStreamBeginCapture(s0_, cudaStreamCaptureModeThreadLocal));
    try {
      enqueue_fn(s0_);
    } catch (...) {
      cudaStreamEndCapture(s0_, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    B2E_CUDA(cudaStreamEndCapture(s0_, &g));
    cudaGraphExec_t ex = nullptr;
    // node priorities (the chains' launch priorities) only apply with this flag
    B2E_CUDA(cudaGraphInstantiate(&ex, g, cudaGraphInstantiateFlagUseNodePriority));
    B2E_CUDA(cudaGraphDestroy(g));
    it = graphs_.emplace(key, ex).first;
  }
  B2E_CUDA(cudaGraphLaunch(it->second, s));
}

// Graph keys: (bucket, set, segment); segment 0 the whole step, 1 the input
// projection of a pipelined step, 2-5 its towers.
static long long graph_key(int rows, int b, int seg) { return ((long long)rows * 8 + b) * 8 + seg; }

bool Engine::pipelined(int n) const { return opt_.pipeline && lanes_for(bucket(n)) == 1; }

void Engine::launch_pipelined(int n, int b) {
  const int rows = bucket(n);
  IoSet& io = io_[b];
  const int P = d_.P, lp = opt_.lp;
  replay(graph_key(rows, b, 1), s_head_, [&](cudaStream_t s) { enqueue_head(rows, b, s); });
  B2E_CUDA(cudaEventRecord(io.head, s_head_));
  for (int t = 0; t < 4; ++t) {
    Chain& ch = chains_[t];
    // the chain's stream already holds this tower's previous step: the state
    // rows it wrote are final before this step's kernels read them
    B2E_CUDA(cudaStreamWaitEvent(ch.s, io.head, 0));
    replay(graph_key(rows, b, 2 + t), ch.s, [&](cudaStream_t s) {
      const StepCtx c = chain_ctx(t, s, rows, io.d_n, io.d_slots);
      const void* up = static_cast<const uint8_t*>(io.d_up) + size_t(t) * P * dtype_size(lp);
      tower_forward(towers_[t], ch, t, c, up, 4 * P, io.d_preds);
    });
    B2E_CUDA(cudaEventRecord(io.tower[t], ch.s));
  }
  for (int t = 0; t < 4; ++t) B2E_CUDA(cudaStreamWaitEvent(s0_, io.tower[t], 0));
}

void Engine::launch(int n, int b, cudaStream_t s) {
  const int rows = bucket(n);
  replay(graph_key(rows, b, 0), s, [&](cudaStream_t cs) { enqueue(rows, b, cs); });
}

void Engine::order_after_last_step(cudaStream_t s) {
  // always, even on the stream it was recorded on: a stream handle may have been
  // destroyed and handed out again since
  if (last_stream_) B2E_CUDA(cudaStreamWaitEvent(s, last_step_, 0));
}

void Engine::drain() { B2E_CUDA(cudaDeviceSynchronize()); }

int Engine::launches_per_step(int n) {
  if (n <= latency_rows()) return 1;
  B2E_CUDA(cudaSetDevice(opt_.device));
  cudaGraph_t g = nullptr;
  B2E_CUDA(cudaStreamBeginCapture(s0_, cudaStreamCaptureModeThreadLocal));
  try {
    enqueue(bucket(n), 0, s0_);
  } catch (...) {
    cudaStreamEndCapture(s0_, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  B2E_CUDA(cudaStreamEndCapture(s0_, &g));
  size_t count = 0;
  B2E_CUDA(cudaGraphGetNodes(g, nullptr, &count));
  std::vector<cudaGraphNode_t> nodes(count);
  B2E_CUDA(cudaGraphGetNodes(g, nodes.data(), &count));
  int kernels = 0;
  for (auto& nd : nodes) {
    cudaGraphNodeType ty;
    B2E_CUDA(cudaGraphNodeGetType(nd, &ty));
    if (ty == cudaGraphNodeTypeKernel) ++kernels;
  }
  B2E_CUDA(cudaGraphDestroy(g));
  return kernels;
}

void Engine::check_host_slots(const int* slots, int n) {
  B2E_CHECK(n >= 1 && n <= opt_.max_batch, kErrCapacity,
            "batch of " + std::to_string(n) + " rows is outside 1.." + std::to_string(opt_.max_batch));
  B2E_CHECK(slots != nullptr, kErrInvalid, "null slot array");
  int i = 0;
  for (; i < n; ++i) {
    const int s = slots[i];
    if (s < 0 || s >= opt_.capacity || seen_[s]) break;
    seen_[s] = 1;
  }
  for (int j = 0; j < i; ++j) seen_[slots[j]] = 0;
  if (i < n) {
    const int s = slots[i];
    B2E_CHECK(!(s < 0 || s >= opt_.capacity), kErrCapacity, "slot " + std::to_string(s) + " outside the state table");
    throw Error(kErrInvalid, "slot " + std::to_string(s) + " appears twice in one step");
  }
}

void Engine::submit(const int* slots, const float* feats, int n) {
  B2E_CHECK(int(host_fifo_.size()) < kSets, kErrInvalid,
            "two host steps are already in flight on this engine: wait() for one first");
  check_host_slots(slots, n);
  B2E_CHECK(feats != nullptr, kErrInvalid, "null feature array");
  B2E_CUDA(cudaSetDevice(opt_.device));
  const int b = next_set_;
  next_set_ = (next_set_ + 1) % kSets;
  IoSet& io = io_[b];
  if (io.used) B2E_CUDA(cudaEventSynchronize(io.done));  // its pinned buffers are free
  const int F = d_.F;
  if (n <= latency_rows()) {
    // one kernel: the rows travel as launch parameters, the predictions and
    // the error word land straight in the set's pinned buffer
    LatIO li{};
    li.n = n;
    std::memcpy(li.slots, slots, size_t(n) * 4);
    std::memcpy(li.feats, feats, size_t(n) * F * 4);
    li.preds = reinterpret_cast<float*>(io.h_io + preds_off_);
    li.err_out = reinterpret_cast<int*>(io.h_io + err_off_);
    order_after_last_step(s0_);
    lat_->launch(li, s0_);
    B2E_CUDA(cudaEventRecord(io.stepped, s0_));
    B2E_CUDA(cudaEventRecord(last_step_, s0_));
    last_stream_ = s0_;
    last_pipelined_ = false;
    B2E_CUDA(cudaEventRecord(io.done, s0_));
    io.used = true;
    io.host_n = n;
    host_fifo_.push_back(b);
    return;
  }
  std::memcpy(io.h_io, &n, 4);
  std::memcpy(io.h_io + slots_off_, slots, size_t(n) * 4);
  std::memcpy(io.h_io + feats_off_, feats, size_t(n) * F * 4);
  // inputs on their own stream: they land while the step before still runs
  B2E_CUDA(cudaMemcpyAsync(io.d_io, io.h_io, 4, cudaMemcpyHostToDevice, s_h2d_));
  B2E_CUDA(cudaMemcpyAsync(io.d_slots, io.h_io + slots_off_, size_t(n) * 4, cudaMemcpyHostToDevice, s_h2d_));
  B2E_CUDA(cudaMemcpyAsync(io.d_feats, io.h_io + feats_off_, size_t(n) * F * 4, cudaMemcpyHostToDevice, s_h2d_));
  B2E_CUDA(cudaEventRecord(io.in_ready, s_h2d_));
  if (pipelined(n)) {
    // the set's previous step finished before this submit (io.done above)
    B2E_CUDA(cudaStreamWaitEvent(s_head_, io.in_ready, 0));
    if (!last_pipelined_) order_after_last_step(s_head_);
    launch_pipelined(n, b);
  } else {
    order_after_last_step(s0_);
    B2E_CUDA(cudaStreamWaitEvent(s0_, io.in_ready, 0));
    launch(n, b, s0_);
  }
  B2E_CUDA(cudaEventRecord(io.stepped, s0_));
  B2E_CUDA(cudaEventRecord(last_step_, s0_));
  last_stream_ = s0_;
  last_pipelined_ = pipelined(n);
  // predictions out on their own stream: the next step's graph does not wait for them
  B2E_CUDA(cudaStreamWaitEvent(s_d2h_, io.stepped, 0));
  B2E_CUDA(cudaMemcpyAsync(io.h_io + preds_off_, io.d_preds, size_t(n) * 16, cudaMemcpyDeviceToHost, s_d2h_));
  B2E_CUDA(cudaMemcpyAsync(io.h_io + err_off_, d_err_, 4, cudaMemcpyDeviceToHost, s_d2h_));
  B2E_CUDA(cudaEventRecord(io.done, s_d2h_));
  io.used = true;
  io.host_n = n;
  host_fifo_.push_back(b);
}

void Engine::wait(float* preds) {
  B2E_CHECK(!host_fifo_.empty(), kErrInvalid, "no step in flight");
  const int b = host_fifo_.front();
  host_fifo_.erase(host_fifo_.begin());
  IoSet& io = io_[b];
  const int n = io.host_n;
  io.host_n = -1;
  B2E_CUDA(cudaSetDevice(opt_.device));
  B2E_CUDA(cudaEventSynchronize(io.done));
  if (preds) std::memcpy(preds, io.h_io + preds_off_, size_t(n) * 16);
  int err = 0;
  std::memcpy(&err, io.h_io + err_off_, 4);
  if (err != 0)
    throw Error(kErrDevice, "device error word " + std::to_string(err) +
                                " after this step (101-103: a tensor-core wait timed out; 1: slots outside the "
                                "table): its predictions and state are not valid; b2e_engine_device_error clears it");
}

void Engine::step_device(const int* d_slots, const float* d_feats, int n, float* d_preds, cudaStream_t s) {
  B2E_CHECK(host_fifo_.empty(), kErrInvalid, "a host step is in flight on this engine");
  B2E_CHECK(n >= 1 && n <= opt_.max_batch, kErrCapacity, "batch outside 1..max_batch");
  B2E_CHECK(d_slots && d_feats && d_preds, kErrInvalid, "null device buffer");
  B2E_CUDA(cudaSetDevice(opt_.device));
  IoSet& io = io_[0];
  order_after_last_step(s);
  if (io.used) B2E_CUDA(cudaStreamWaitEvent(s, io.done, 0));
  B2E_CUDA(cudaMemcpyAsync(io.d_slots, d_slots, size_t(n) * 4, cudaMemcpyDeviceToDevice, s));
  B2E_CUDA(cudaMemcpyAsync(io.d_feats, d_feats, size_t(n) * d_.F * 4, cudaMemcpyDeviceToDevice, s));
  k_validate<<<1, 1024, 0, s>>>(io.d_slots, n, opt_.capacity, io.d_n, d_err_);
  B2E_CUDA(cudaGetLastError());
  launch(n, 0, s);
  B2E_CUDA(cudaMemcpyAsync(d_preds, io.d_preds, size_t(n) * 16, cudaMemcpyDeviceToDevice, s));
  B2E_CUDA(cudaEventRecord(io.done, s));
  B2E_CUDA(cudaEventRecord(last_step_, s));
  last_stream_ = s;
  last_pipelined_ = false;
  io.used = true;
}

void Engine::submit_device(const int* d_slots, const float* d_feats, int n, float* d_preds, cudaStream_t s) {
  B2E_CHECK(host_fifo_.empty(), kErrInvalid, "a host step is in flight on this engine");
  B2E_CHECK(n >= 1 && n <= opt_.max_batch, kErrCapacity, "batch outside 1..max_batch");
  B2E_CHECK(d_slots && d_feats && d_preds, kErrInvalid, "null device buffer");
  B2E_CUDA(cudaSetDevice(opt_.device));
  const int b = next_set_;
  next_set_ = (next_set_ + 1) % kSets;
  IoSet& io = io_[b];
  const bool pipe = pipelined(n);
  // inputs: after the caller's work on `s`; the set: after its previous step's
  // predictions were copied out
  B2E_CUDA(cudaEventRecord(io.in_ready, s));
  B2E_CUDA(cudaStreamWaitEvent(s_head_, io.in_ready, 0));
  if (io.used) B2E_CUDA(cudaStreamWaitEvent(s_head_, io.done, 0));
  if (!pipe || !last_pipelined_) order_after_last_step(s_head_);
  B2E_CUDA(cudaMemcpyAsync(io.d_slots, d_slots, size_t(n) * 4, cudaMemcpyDeviceToDevice, s_head_));
  B2E_CUDA(cudaMemcpyAsync(io.d_feats, d_feats, size_t(n) * d_.F * 4, cudaMemcpyDeviceToDevice, s_head_));
  k_validate<<<1, 1024, 0, s_head_>>>(io.d_slots, n, opt_.capacity, io.d_n, d_err_);
  B2E_CUDA(cudaGetLastError());
  if (pipe) {
    launch_pipelined(n, b);
  } else {
    B2E_CUDA(cudaEventRecord(io.head, s_head_));
    B2E_CUDA(cudaStreamWaitEvent(s0_, io.head, 0));
    launch(n, b, s0_);
  }
  B2E_CUDA(cudaMemcpyAsync(d_preds, io.d_preds, size_t(n) * 16, cudaMemcpyDeviceToDevice, s0_));
  B2E_CUDA(cudaEventRecord(io.stepped, s0_));
  B2E_CUDA(cudaEventRecord(io.done, s0_));
  B2E_CUDA(cudaEventRecord(last_step_, s0_));
  last_stream_ = s0_;
  last_pipelined_ = pipe;
  io.used = true;
}

void Engine::join_device(cudaStream_t s) {
  B2E_CUDA(cudaSetDevice(opt_.device));
  order_after_last_step(s);
}

int Engine::device_error() {
  B2E_CUDA(cudaSetDevice(opt_.device));
  drain();
  int e = 0;
  B2E_CUDA(cudaMemcpy(&e, d_err_, 4, cudaMemcpyDeviceToHost));
  B2E_CUDA(cudaMemset(d_err_, 0, 4));
  return e;
}

void Engine::reset_slots(const int* slots, int n) {
  B2E_CHECK(host_fifo_.empty(), kErrInvalid, "a step is in flight on this engine");
  B2E_CUDA(cudaSetDevice(opt_.device));
  drain();
  for (int i0 = 0; i0 < n; i0 += opt_.max_batch) {
    const int m = std::min(opt_.max_batch, n - i0);
    for (int i = 0; i < m; ++i)
      B2E_CHECK(slots[i0 + i] >= 0 && slots[i0 + i] < opt_.capacity, kErrCapacity, "slot outside the state table");
    std::memcpy(h_rs_, slots + i0, size_t(m) * 4);
    B2E_CUDA(cudaMemcpyAsync(d_rs_, h_rs_, size_t(m) * 4, cudaMemcpyHostToDevice, s0_));
    arena_.reset_slots(d_rs_, m, s0_);
    B2E_CUDA(cudaStreamSynchronize(s0_));
  }
}

void Engine::read_slot(int slot, void* host) {
  B2E_CHECK(host_fifo_.empty(), kErrInvalid, "a step is in flight on this engine");
  B2E_CUDA(cudaSetDevice(opt_.device));
  drain();
  arena_.read_slot(slot, host);
}

void Engine::write_slot(int slot, const void* host) {
  B2E_CHECK(host_fifo_.empty(), kErrInvalid, "a step is in flight on this engine");
  B2E_CUDA(cudaSetDevice(opt_.device));
  drain();
  arena_.write_slot(slot, host);
}

}  // namespace b2e
