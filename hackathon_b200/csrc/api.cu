// C ABI (include/b2e.h): status codes in, exceptions never cross the boundary.
#include <cstring>
#include <functional>
#include <memory>
#include <string>

#include "../../include/b2e.h"
#include "cells.cuh"
#include "engine.cuh"
#include "gemm.cuh"
#include "stream.cuh"

using namespace b2e;

struct b2e_engine {
  std::unique_ptr<Engine> eng;
};

struct b2e_layer {
  Dims d;
  int kind = 0, device = 0, capacity = 0, max_batch = 0, lp = 0;
  bool pdl = true;
  WeightPack pack;
  StateArena arena;
  std::unique_ptr<Layer> layer;
  uint8_t* scratch = nullptr;
  void* x_lp = nullptr;  // the step's input in the CastLinear type (low-precision weights only)
  int* d_n = nullptr;
  int* d_err = nullptr;
  ~b2e_layer() {
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    if (scratch) cudaFree(scratch);
    if (x_lp) cudaFree(x_lp);
    if (d_n) cudaFree(d_n);
  }
};

namespace {

thread_local std::string g_err;

template <class F>
int guard(F&& f) {
  try {
    f();
    return B2E_OK;
  } catch (const Error& e) {
    g_err = e.what();
    return e.code;
  } catch (const std::bad_alloc&) {
    g_err = "host allocation failed";
    return B2E_ERR_INTERNAL;
  } catch (const std::exception& e) {
    g_err = e.what();
    return B2E_ERR_INTERNAL;
  }
}

Dims to_dims(const b2e_model_config* c) {
  B2E_CHECK(c != nullptr, kErrInvalid, "null model config");
  Dims d;
  d.H = c->hidden_size;
  d.P = c->proj_size;
  d.depth = c->tower_depth;
  d.heads = c->num_heads;
  d.F = c->num_features;
  d.m_hs = c->mamba_head_size > 0 ? c->mamba_head_size : 64;
  d.m_bc = c->mamba_bc_size > 0 ? c->mamba_bc_size : 128;
  return d;
}

EngineOptions to_opts(const b2e_engine_options* o) {
  B2E_CHECK(o != nullptr, kErrInvalid, "null engine options");
  EngineOptions e;
  e.device = o->device;
  e.lp = o->linear_dtype;
  e.capacity = o->capacity;
  e.max_batch = o->max_batch;
  e.graphs = o->use_graphs != 0;
  if (o->lanes > 0) e.lanes = o->lanes;
  if (o->lane_min_rows > 0) e.lane_min_rows = o->lane_min_rows;
  if (o->lane_towers != 0) e.lane_towers = o->lane_towers;
  e.pdl = !(o->flags & B2E_FLAG_NO_PDL);
  e.priorities = !(o->flags & B2E_FLAG_NO_PRIORITIES);
  e.latency = !(o->flags & B2E_FLAG_NO_LATENCY_PATH);
  e.pipeline = !(o->flags & B2E_FLAG_NO_PIPELINE);
  return e;
}

void fill_source(WeightSource& src, const b2e_tensor* t, int32_t n) {
  B2E_CHECK(n >= 0 && (n == 0 || t != nullptr), kErrInvalid, "null tensor list");
  for (int32_t i = 0; i < n; ++i) {
    B2E_CHECK(t[i].name != nullptr, kErrInvalid, "tensor without a name");
    src.add(t[i].name, t[i].data, t[i].numel);
  }
}

Engine& E(b2e_engine* e) {
  B2E_CHECK(e && e->eng, kErrInvalid, "null engine");
  return *e->eng;
}

b2e_layer& L(b2e_layer* l) {
  B2E_CHECK(l && l->layer, kErrInvalid, "null layer");
  return *l;
}

__global__ void k_validate_slots(const int* slots, int n, int capacity, int* n_dev, int* err) {
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

// x rounded to the CastLinear type, rows < *n_dev: the cast CastLinear.forward
// applies to its input (example_model.py:93-94). A layer whose first projection
// reads it runs that GEMM with same-type operands (the tensor-core path).
__global__ void k_layer_in_lp(const float* x, int H, int lp, void* out, const int* n_dev) {
  const long long total = (long long)(*n_dev) * H;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x)
    store_as(lp, out, size_t(i), x[i]);
}

void check_cell(int batch, int heads, int a, int b) {
  B2E_CHECK(batch >= 0 && batch <= 65535, kErrInvalid, "batch must be in 0..65535");
  B2E_CHECK(heads > 0 && a > 0 && b > 0, kErrInvalid, "cell sizes must be positive");
}

}  // namespace

namespace b2e {
// The status/last-error translation above, for entry points defined in other
// translation units.
int abi_call(const std::function<void()>& f) { return guard(f); }
}  // namespace b2e

extern "C" {

const char* b2e_last_error(void) { return g_err.c_str(); }
const char* b2e_version(void) { return "b2e 0.1 sm_100a"; }

int b2e_engine_create(const b2e_model_config* cfg, const b2e_engine_options* opt, const b2e_tensor* tensors,
                      int32_t n_tensors, b2e_engine** out) {
  return guard([&] {
    B2E_CHECK(out != nullptr, kErrInvalid, "null output handle");
    *out = nullptr;
    WeightSource src;
    fill_source(src, tensors, n_tensors);
    auto h = std::make_unique<b2e_engine>();
    h->eng = std::make_unique<Engine>(to_dims(cfg), to_opts(opt), src);
    *out = h.release();
  });
}

void b2e_engine_destroy(b2e_engine* e) { delete e; }

int b2e_engine_step(b2e_engine* e, const int32_t* slots, const float* features, int32_t n, float* preds) {
  return guard([&] {
    B2E_CHECK(preds != nullptr, kErrInvalid, "null prediction buffer");
    E(e).step(slots, features, n, preds);
  });
}

int b2e_engine_submit(b2e_engine* e, const int32_t* slots, const float* features, int32_t n) {
  return guard([&] { E(e).submit(slots, features, n); });
}

int b2e_engine_wait(b2e_engine* e, float* preds) {
  return guard([&] { E(e).wait(preds); });
}

int b2e_engine_step_device(b2e_engine* e, const int32_t* d_slots, const float* d_features, int32_t n,
                           float* d_preds, void* stream) {
  return guard([&] { E(e).step_device(d_slots, d_features, n, d_preds, static_cast<cudaStream_t>(stream)); });
}

int b2e_set_state_kernel_waves(int32_t waves, int32_t* previous) {
  return guard([&] {
    B2E_CHECK(waves >= 0 && waves <= 64, kErrInvalid, "state kernel waves must be in 0..64");
    const int old = set_state_kernel_waves(waves);
    if (previous) *previous = old;
  });
}

int b2e_engine_submit_device(b2e_engine* e, const int32_t* d_slots, const float* d_features, int32_t n,
                             float* d_preds, void* stream) {
  return guard([&] { E(e).submit_device(d_slots, d_features, n, d_preds, static_cast<cudaStream_t>(stream)); });
}

int b2e_engine_join_device(b2e_engine* e, void* stream) {
  return guard([&] { E(e).join_device(static_cast<cudaStream_t>(stream)); });
}

int b2e_engine_device_error(b2e_engine* e, int32_t* flag) {
  return guard([&] {
    B2E_CHECK(flag != nullptr, kErrInvalid, "null flag");
    *flag = E(e).device_error();
  });
}

int b2e_engine_reset_slots(b2e_engine* e, const int32_t* slots, int32_t n) {
  return guard([&] {
    B2E_CHECK(n >= 0 && (n == 0 || slots), kErrInvalid, "null slot array");
    E(e).reset_slots(slots, n);
  });
}

int b2e_engine_slot_bytes(const b2e_engine* e, int64_t* bytes) {
  return guard([&] {
    B2E_CHECK(e && e->eng && bytes, kErrInvalid, "null argument");
    *bytes = int64_t(e->eng->slot_bytes());
  });
}

int b2e_engine_read_slot(b2e_engine* e, int32_t slot, void* host, int64_t bytes) {
  return guard([&] {
    B2E_CHECK(host && bytes == int64_t(E(e).slot_bytes()), kErrInvalid, "slot buffer has the wrong size");
    E(e).read_slot(slot, host);
  });
}

int b2e_engine_write_slot(b2e_engine* e, int32_t slot, const void* host, int64_t bytes) {
  return guard([&] {
    B2E_CHECK(host && bytes == int64_t(E(e).slot_bytes()), kErrInvalid, "slot buffer has the wrong size");
    E(e).write_slot(slot, host);
  });
}

int b2e_engine_launches(b2e_engine* e, int32_t n, int32_t* kernels) {
  return guard([&] {
    B2E_CHECK(kernels != nullptr, kErrInvalid, "null output");
    B2E_CHECK(n >= 1 && n <= E(e).max_batch(), kErrCapacity, "batch outside 1..max_batch");
    *kernels = E(e).launches_per_step(n);
  });
}

int b2e_engine_latency_rows(b2e_engine* e, int32_t* rows, int32_t* cluster) {
  return guard([&] {
    B2E_CHECK(rows != nullptr, kErrInvalid, "null output");
    *rows = E(e).latency_rows();
    if (cluster) *cluster = E(e).latency_cluster();
  });
}

int b2e_engine_memory(const b2e_engine* e, int64_t* weight_bytes, int64_t* state_bytes) {
  return guard([&] {
    B2E_CHECK(e && e->eng, kErrInvalid, "null engine");
    if (weight_bytes) *weight_bytes = int64_t(e->eng->weight_bytes());
    if (state_bytes) *state_bytes = int64_t(e->eng->state_bytes());
  });
}

int b2e_mlstm_step(float* cell, const float* q, const float* k, const float* v, const float* i_gate,
                   const float* f_gate, const uint8_t* mask, int32_t batch, int32_t heads, int32_t size_h,
                   int32_t size_k, float* out, void* stream) {
  return guard([&] {
    check_cell(batch, heads, size_h, size_k);
    B2E_CHECK(cell && q && k && v && i_gate && f_gate && out, kErrInvalid, "null operand");
    OuterRowsParams p;
    p.at = {cell, (long long)heads * size_h * size_k, nullptr, mask, batch, nullptr};
    p.nh = heads; p.sh = size_h; p.sk = size_k;
    p.f = f_gate; p.f_rs = heads; p.f_hs = 1;
    p.i = i_gate; p.i_rs = heads; p.i_hs = 1;
    p.kv = k; p.k_rs = heads * size_h;
    p.v = v; p.v_rs = heads * size_k;
    p.q = q; p.q_rs = heads * size_h;
    p.out = out; p.o_rs = heads * size_k;
    outer_rows(p, batch, static_cast<cudaStream_t>(stream));
  });
}

int b2e_retnet_step(float* state, const float* k_rope, const float* v, const float* q_scaled, const float* decay,
                    const uint8_t* mask, int32_t batch, int32_t heads, int32_t size_h, int32_t size_k, float* out,
                    void* stream) {
  return guard([&] {
    check_cell(batch, heads, size_h, size_k);
    B2E_CHECK(state && k_rope && v && q_scaled && decay && out, kErrInvalid, "null operand");
    OuterRowsParams p;
    p.at = {state, (long long)heads * size_h * size_k, nullptr, mask, batch, nullptr};
    p.nh = heads; p.sh = size_h; p.sk = size_k;
    p.f = decay; p.f_rs = 0; p.f_hs = 1;
    p.kv = k_rope; p.k_rs = heads * size_h;
    p.v = v; p.v_rs = heads * size_k;
    p.q = q_scaled; p.q_rs = heads * size_h;
    p.out = out; p.o_rs = heads * size_k;
    outer_rows(p, batch, static_cast<cudaStream_t>(stream));
  });
}

int b2e_mamba2_step(float* ssm, const float* x, const float* b, const float* c, const float* dt,
                    const float* decay, const uint8_t* mask, int32_t batch, int32_t heads, int32_t size_h,
                    int32_t size_c, float* out, void* stream) {
  return guard([&] {
    check_cell(batch, heads, size_h, size_c);
    B2E_CHECK(ssm && x && b && c && dt && decay && out, kErrInvalid, "null operand");
    SsmColsParams p;
    p.at = {ssm, (long long)heads * size_h * size_c, nullptr, mask, batch, nullptr};
    p.nh = heads; p.sh = size_h; p.sc = size_c;
    p.x = x; p.x_rs = heads * size_h;
    p.b = b; p.b_rs = size_c;
    p.c = c; p.c_rs = size_c;
    p.dt = dt; p.dt_rs = heads;
    p.decay = decay; p.dc_rs = heads;
    p.out = out; p.o_rs = heads * size_h;
    ssm_cols(p, batch, static_cast<cudaStream_t>(stream));
  });
}

int b2e_linear(const void* x, int32_t x_dtype, int32_t m, int32_t k, const void* w, int32_t w_dtype,
               const void* bias, int32_t n, int32_t act, float* y, int32_t* d_err, void* stream) {
  return guard([&] {
    B2E_CHECK(x && w && y, kErrInvalid, "null operand");
    B2E_CHECK(m > 0 && m <= 65535 * 64 && n > 0 && k > 0, kErrInvalid, "bad GEMM sizes");
    B2E_CHECK(w_dtype == kF32 || w_dtype == kBF16 || w_dtype == kF16, kErrInvalid, "unknown weight dtype");
    B2E_CHECK(x_dtype == kF32 || x_dtype == w_dtype, kErrInvalid, "x must be f32 or the weight's dtype");
    B2E_CHECK(act == kActNone || act == kActRelu, kErrInvalid, "unknown activation");
    gemm_tc_init();
    GemmParams p;
    p.g[0].A = x;
    p.g[0].W = w;
    p.g[0].bias = bias;
    p.g[0].C = y;
    p.M_max = m;
    p.N = n;
    p.K = k;
    p.lda = k;
    p.ldw = k;
    p.ldc = n;
    p.a_type = x_dtype;
    p.w_type = w_dtype;
    p.bias_type = w_dtype;
    p.round_out = w_dtype != kF32;
    p.act = act;
    p.err = d_err;
    gemm(p, static_cast<cudaStream_t>(stream));
  });
}

int b2e_layer_create(int32_t kind, const b2e_model_config* cfg, const b2e_engine_options* opt,
                     const b2e_tensor* tensors, int32_t n_tensors, b2e_layer** out) {
  return guard([&] {
    B2E_CHECK(out != nullptr, kErrInvalid, "null output handle");
    *out = nullptr;
    const EngineOptions o = to_opts(opt);
    B2E_CHECK(o.capacity > 0 && o.max_batch > 0 && o.max_batch <= 65535, kErrInvalid, "bad capacity or max_batch");
    auto h = std::make_unique<b2e_layer>();
    h->d = to_dims(cfg);
    h->d.validate();
    h->kind = kind;
    h->device = o.device;
    h->capacity = o.capacity;
    h->max_batch = o.max_batch;
    h->lp = o.lp;
    h->pdl = o.pdl;
    B2E_CUDA(cudaSetDevice(o.device));
    gemm_tc_init();
    stream_init();
    WeightSource src;
    fill_source(src, tensors, n_tensors);
    h->layer = Layer::make(kind, h->d, o.lp);
    h->layer->load(src, h->pack, "");
    src.check_all_used();
    h->pack.upload();
    h->layer->declare_state(h->arena);
    h->arena.allocate(o.capacity);
    h->layer->resolve(h->pack, h->arena);
    B2E_CUDA(cudaMalloc(&h->scratch, h->layer->scratch_bytes(o.max_batch) + 256));
    // the xLSTM layer's first projections read normalised rows it computes itself
    if (o.lp != kF32 && kind != kXLSTM) B2E_CUDA(cudaMalloc(&h->x_lp, size_t(o.max_batch) * h->d.H * dtype_size(o.lp)));
    B2E_CUDA(cudaMalloc(&h->d_n, 16));
    h->d_err = h->d_n + 1;
    B2E_CUDA(cudaMemset(h->d_n, 0, 16));
    h->arena.reset_all(nullptr);
    B2E_CUDA(cudaDeviceSynchronize());
    *out = h.release();
  });
}

void b2e_layer_destroy(b2e_layer* l) { delete l; }

int b2e_layer_step_device(b2e_layer* l, const int32_t* d_slots, const float* d_x, int32_t n, float* d_y,
                          void* stream) {
  return guard([&] {
    b2e_layer& h = L(l);
    B2E_CHECK(n >= 1 && n <= h.max_batch, kErrCapacity, "batch outside 1..max_batch");
    B2E_CHECK(d_slots && d_x && d_y, kErrInvalid, "null device buffer");
    B2E_CUDA(cudaSetDevice(h.device));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    k_validate_slots<<<1, 1024, 0, s>>>(d_slots, n, h.capacity, h.d_n, h.d_err);
    B2E_CUDA(cudaGetLastError());
    StepCtx c;
    c.s = s;
    c.rows = n;
    c.n_dev = h.d_n;
    c.slots = d_slots;
    c.lp = h.lp;
    c.err = h.d_err;
    c.ln.pdl = c.ln_bulk.pdl = h.pdl;
    if (h.x_lp) {
      const int blocks = std::max(1, std::min(ceil_div(long(n) * h.d.H, 256 * 4), 148 * 8));
      k_layer_in_lp<<<blocks, 256, 0, s>>>(d_x, h.d.H, h.lp, h.x_lp, h.d_n);
      B2E_CUDA(cudaGetLastError());
    }
    h.layer->forward(c, d_x, h.x_lp, d_y, nullptr, h.scratch);
  });
}

int b2e_layer_reset_slots(b2e_layer* l, const int32_t* slots, int32_t n) {
  return guard([&] {
    b2e_layer& h = L(l);
    B2E_CHECK(n >= 0 && (n == 0 || slots), kErrInvalid, "null slot array");
    B2E_CUDA(cudaSetDevice(h.device));
    for (int i = 0; i < n; ++i)
      B2E_CHECK(slots[i] >= 0 && slots[i] < h.capacity, kErrCapacity, "slot outside the state table");
    int* d = nullptr;
    B2E_CUDA(cudaMalloc(&d, size_t(std::max(n, 1)) * 4));
    cudaMemcpy(d, slots, size_t(n) * 4, cudaMemcpyHostToDevice);
    h.arena.reset_slots(d, n, nullptr);
    cudaError_t e = cudaDeviceSynchronize();
    cudaFree(d);
    B2E_CUDA(e);
  });
}

int b2e_layer_slot_bytes(const b2e_layer* l, int64_t* bytes) {
  return guard([&] {
    B2E_CHECK(l && bytes, kErrInvalid, "null argument");
    *bytes = int64_t(l->arena.slot_bytes());
  });
}

int b2e_layer_read_slot(b2e_layer* l, int32_t slot, void* host, int64_t bytes) {
  return guard([&] {
    b2e_layer& h = L(l);
    B2E_CHECK(host && bytes == int64_t(h.arena.slot_bytes()), kErrInvalid, "slot buffer has the wrong size");
    B2E_CUDA(cudaSetDevice(h.device));
    B2E_CUDA(cudaDeviceSynchronize());
    h.arena.read_slot(slot, host);
  });
}

int b2e_layer_write_slot(b2e_layer* l, int32_t slot, const void* host, int64_t bytes) {
  return guard([&] {
    b2e_layer& h = L(l);
    B2E_CHECK(host && bytes == int64_t(h.arena.slot_bytes()), kErrInvalid, "slot buffer has the wrong size");
    B2E_CUDA(cudaSetDevice(h.device));
    B2E_CUDA(cudaDeviceSynchronize());
    h.arena.write_slot(slot, host);
  });
}

}  // extern "C"
