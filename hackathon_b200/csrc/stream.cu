// Bulk-copy streaming state steps (see stream.cuh).
#include "stream.cuh"

#include <algorithm>
#include <atomic>
#include <mutex>

#include "mbarrier.cuh"

namespace b2e {
namespace {

using namespace stream_cfg;
constexpr int kCT = 32 * kCW;                 // compute threads (named barrier 1)
constexpr int kBulkThreads = 32 + kCT;        // + the producer warp
constexpr uint32_t kStageBytes = kStateMax + kOpsMax;
constexpr size_t kRingBytes = size_t(kStages) * kStageBytes;
constexpr size_t kBulkSmem = kStreamSmem;
enum BulkError : int { kBulkTimeoutProducer = 111, kBulkTimeoutConsumer = 112 };

// Shared-memory ring: kStages stages of [state | operands], full/empty barriers,
// the abort flag, the consumers' per-item verdict, and cross-warp partials.
struct Ring {
  uint8_t* base;
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort_flag;
  volatile int* go;
  float4* part;  // [kCW][32]
};

__device__ __forceinline__ Ring ring_setup() {
  extern __shared__ __align__(128) uint8_t sm_raw[];
  uint8_t* sm = sm_raw + ((128u - (smem_u32(sm_raw) & 127u)) & 127u);
  Ring r;
  r.base = sm;
  r.full = reinterpret_cast<uint64_t*>(sm + kRingBytes);
  r.empty = r.full + kStages;
  r.abort_flag = reinterpret_cast<volatile int*>(r.empty + kStages);
  r.go = r.abort_flag + 1;
  r.part = reinterpret_cast<float4*>(sm + kRingBytes + 256);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&r.full[s], 2);  // the producer's expect_tx arrive + its cp.async completion arrive
      mbar_init(&r.empty[s], 1);
    }
    *r.abort_flag = 0;
    *r.go = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  return r;
}

// Producer (one thread): item k of this CTA goes to stage k % kStages once the
// consumers released that stage. `issue(k, stage, bar)` arms `bar` with the
// item's byte count and issues its loads; `issue.prefetch(k)` loads what the
// producer itself must know about item k (its slot) one item ahead.
template <class Issue>
__device__ void produce(const Ring& r, int my, int* err, Issue&& issue) {
  int issued = 0;
  issue.prefetch(0);
  for (int k = 0; k < my; ++k) {
    const int s = k % kStages;
    const uint32_t ph = (k / kStages) & 1;
    if (k >= kStages && !mbar_wait(&r.empty[s], ph ^ 1, r.abort_flag)) {
      if (err && !*r.abort_flag) atomicExch(err, kBulkTimeoutProducer);
      *r.abort_flag = 1;
      break;
    }
    if (*r.abort_flag) break;
    issue(k, r.base + size_t(s) * kStageBytes, &r.full[s]);
    ++issued;
    if (k + 1 < my) issue.prefetch(k + 1);
  }
  if (*r.abort_flag) {
    // every load issued lands before the CTA leaves (bounded)
    volatile int never = 0;
    for (int k = max(0, issued - kStages); k < issued; ++k) mbar_wait(&r.full[k % kStages], (k / kStages) & 1, &never);
  }
}

// Consumers (kCT threads): wait for item k, `compute(k, stage)` in shared
// memory (false: nothing to write back),
// then one thread writes the stage back with `store(k, stage)` (a bulk store)
// and releases the previous item's stage once its store has read it, and every
// consumer runs `after(k, stage, wrote)`: work that needs the whole CTA's
// compute of item k (it sits between the barrier before the store and the next
// item's first barrier, so it costs no barrier of its own). Every consumer
// thread takes the same path through the named barriers.
template <class Compute, class Store, class After>
__device__ void consume(const Ring& r, int my, int* err, int ctid, Compute&& compute, Store&& store, After&& after) {
  for (int k = 0; k < my; ++k) {
    const int s = k % kStages;
    const uint32_t ph = (k / kStages) & 1;
    uint8_t* st = r.base + size_t(s) * kStageBytes;
    if (ctid == 0) {
      const bool ok = mbar_wait(&r.full[s], ph, r.abort_flag);
      if (!ok) {
        if (err && !*r.abort_flag) atomicExch(err, kBulkTimeoutConsumer);
        *r.abort_flag = 1;
      }
      *r.go = ok && !*r.abort_flag;
    }
    named_bar(1, kCT);
    if (!*r.go) break;  // the leader's verdict, the same for every consumer
    mbar_try(&r.full[s], ph);  // completed (the leader saw it): acquires the bulk-loaded bytes for this thread
    const bool wrote = compute(k, st);
    fence_proxy_async();  // this thread's shared-memory writes, visible to the bulk store
    named_bar(1, kCT);
    if (ctid == 0) {
      if (wrote) store(k, st);
      bulk_commit();
      bulk_wait_read<1>();  // the previous item's store has read its stage
      if (k >= 1) mbar_arrive(&r.empty[(k - 1) % kStages]);
    }
    after(k, st, wrote);
  }
  if (ctid == 0) bulk_wait_all();
}

__device__ __forceinline__ long long slot_of(const RowAddr& a, int row) { return a.slots ? a.slots[row] : row; }

// Items of this CTA: chunk == 0 (persistent grid): blockIdx.x, blockIdx.x +
// gridDim.x, ... < items; chunk > 0: [blockIdx.x * chunk, + chunk) < items.
__device__ __forceinline__ int items_of_cta(int items, int chunk) {
  if (chunk > 0) return max(0, min(chunk, items - int(blockIdx.x) * chunk));
  return items > int(blockIdx.x) ? (items - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x) : 0;
}
// The item of this CTA's k-th turn.
__device__ __forceinline__ int item_index(int k, int chunk) {
  return chunk > 0 ? int(blockIdx.x) * chunk + k : int(blockIdx.x) + k * int(gridDim.x);
}

// Per-item scalars (decay factors, gates, the row's mask bit) sit at the end of
// the stage's operand area. The producer writes the mask bit and fetches the
// scalars with 4-byte cp.async copies that complete on the stage's barrier.
constexpr uint32_t kScalarOff = kStateMax + kOpsMax - 128;  // 32 floats
constexpr int kActive = 16;                                 // scalar slot of the row's mask bit
constexpr int kSlot = 24;                                   // scalar slots 24-25: the row's state slot (int64)

// ---- Mamba2: item = (row, head); LC = sc/4 lanes cover one state row p.
struct SsmIssue {
  const SsmColsParams& p;
  int chunk;
  uint32_t sbytes, xb, cb;
  long long slot = 0;  // of the next item, loaded one item ahead
  __device__ void item(int k, int& row, int& h) const {
    const int it = item_index(k, chunk);
    row = it / p.nh;
    h = it - row * p.nh;
  }
  __device__ void prefetch(int k) {
    int row, h;
    item(k, row, h);
    slot = slot_of(p.at, row);
  }
  __device__ void operator()(int k, uint8_t* st, uint64_t* bar) {
    int row, h;
    item(k, row, h);
    float* sc = reinterpret_cast<float*>(st + kScalarOff);
    const bool active = !p.at.mask || p.at.mask[row];
    sc[kActive] = active ? 1.f : 0.f;
    *reinterpret_cast<long long*>(sc + kSlot) = slot;
    if (active) {
      mbar_expect_tx(bar, sbytes + xb + 2 * cb);
      bulk_load_hint(st, p.at.state + slot * p.at.row_stride + size_t(h) * p.sh * p.sc, sbytes, bar, l2_evict_first());
      bulk_load(st + kStateMax, p.x + size_t(row) * p.x_rs + size_t(h) * p.sh, xb, bar);
      bulk_load(st + kStateMax + xb, p.b + size_t(row) * p.b_rs, cb, bar);
      bulk_load(st + kStateMax + xb + cb, p.c + size_t(row) * p.c_rs, cb, bar);
      cp_async4(&sc[0], p.dt + size_t(row) * p.dt_rs + h);
      cp_async4(&sc[1], p.decay + size_t(row) * p.dc_rs + h);
    } else {
      mbar_expect_tx(bar, 0);  // idle row: nothing to load
    }
    cp_async_arrive(bar);
  }
};

template <int LC>
__global__ void __launch_bounds__(kBulkThreads, 2) ssm_bulk_kernel(const __grid_constant__ SsmColsParams p, int chunk) {
  const Ring r = ring_setup();
  pdl_wait();
  const int items = live_rows(p.at.n_dev, p.at.n_host) * p.nh;
  const int my = items_of_cta(items, chunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  SsmIssue is{p, chunk, uint32_t(p.sh) * p.sc * 4, uint32_t(p.sh) * 4, uint32_t(p.sc) * 4};
  if (warp == 0) {
    if (lane == 0) produce(r, my, p.err, is);
    return;
  }
  const uint32_t sbytes = is.sbytes, xb = is.xb, cb = is.cb;
  // A state row (LC float4) is covered by LR lanes holding Q = LC/LR vectors
  // each; a warp takes RPW = 32/LR rows per step.
  constexpr int LR = LC < 8 ? LC : 8, Q = LC / LR, RPW = 32 / LR;
  const int cw = warp - 1, c0 = lane % LR, rsub = lane / LR;
  consume(
      r, my, p.err, threadIdx.x - 32,
      [&](int k, uint8_t* st) -> bool {
        int row, h;
        is.item(k, row, h);
        const float* sc = reinterpret_cast<const float*>(st + kScalarOff);
        float* out = p.out + size_t(row) * p.o_rs + size_t(h) * p.sh;
        if (sc[kActive] == 0.f) {  // idle row: state untouched, output zero
          for (int i = threadIdx.x - 32; i < p.sh; i += kCT) out[i] = 0.f;
          return false;
        }
        float4* H = reinterpret_cast<float4*>(st);
        const float* xs = reinterpret_cast<const float*>(st + kStateMax);
        const float dt = sc[0], dc = sc[1];
        float4 db[Q], cv[Q];  // dt*b and c at this lane's columns c0 + LR*q
#pragma unroll
        for (int q = 0; q < Q; ++q) {
          const float4 b4 = reinterpret_cast<const float4*>(st + kStateMax + xb)[c0 + LR * q];
          db[q] = make_float4(dt * b4.x, dt * b4.y, dt * b4.z, dt * b4.w);
          cv[q] = reinterpret_cast<const float4*>(st + kStateMax + xb + cb)[c0 + LR * q];
        }
        for (int base = cw * RPW; base < p.sh; base += kCW * RPW) {  // warp-uniform
          const int pp = base + rsub;
          const bool ok = pp < p.sh;
          float dot = 0.f;
          if (ok) {
            const float xp = xs[pp];
#pragma unroll
            for (int q = 0; q < Q; ++q) {
              float4* hp = H + pp * LC + c0 + LR * q;
              const float4 cur = *hp;
              float4 nv;  // decay*h + (dt*b)*x  (model/kernels.py:163-171)
              nv.x = fmaf(dc, cur.x, db[q].x * xp);
              nv.y = fmaf(dc, cur.y, db[q].y * xp);
              nv.z = fmaf(dc, cur.z, db[q].z * xp);
              nv.w = fmaf(dc, cur.w, db[q].w * xp);
              *hp = nv;
              dot += fmaf(cv[q].w, nv.w, fmaf(cv[q].z, nv.z, fmaf(cv[q].y, nv.y, cv[q].x * nv.x)));
            }
          }
#pragma unroll
          for (int o = LR / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
          if (ok && c0 == 0) out[pp] = dot;
        }
        return true;
      },
      [&](int k, uint8_t* st) {
        int row, h;
        is.item(k, row, h);
        const long long slot = *reinterpret_cast<const long long*>(reinterpret_cast<const float*>(st + kScalarOff) + kSlot);
        bulk_store_hint(p.at.state + slot * p.at.row_stride + size_t(h) * p.sh * p.sc, st, sbytes, l2_evict_first());
      },
      [](int, uint8_t*, bool) {});
}

// ---- mLSTM / RetNet: item = (row, group of hg heads, hg | kCW); L = sk/4 lanes
// cover one state row; the kCW/hg warps of a head split its rows, and the sum
// over rows closes with shuffles inside a warp and over the head's warps through
// shared memory.
struct OuterIssue {
  const OuterRowsParams& p;
  int chunk;
  int hg, groups;
  uint32_t sbytes, qb, vb;
  long long slot = 0;
  __device__ void item(int k, int& row, int& h0) const {
    const int it = item_index(k, chunk);
    row = it / groups;
    h0 = (it - row * groups) * hg;
  }
  __device__ void prefetch(int k) {
    int row, h0;
    item(k, row, h0);
    slot = slot_of(p.at, row);
  }
  __device__ void operator()(int k, uint8_t* st, uint64_t* bar) {
    int row, h0;
    item(k, row, h0);
    float* sc = reinterpret_cast<float*>(st + kScalarOff);
    const bool active = !p.at.mask || p.at.mask[row];
    sc[kActive] = active ? 1.f : 0.f;
    *reinterpret_cast<long long*>(sc + kSlot) = slot;
    if (active) {
      mbar_expect_tx(bar, sbytes + 2 * qb + vb);
      bulk_load_hint(st, p.at.state + slot * p.at.row_stride + size_t(h0) * p.sh * p.sk, sbytes, bar, l2_evict_first());
      uint8_t* o = st + kStateMax;
      bulk_load(o, p.q + size_t(row) * p.q_rs + size_t(h0) * p.sh, qb, bar);
      bulk_load(o + qb, p.kv + size_t(row) * p.k_rs + size_t(h0) * p.sh, qb, bar);
      bulk_load(o + 2 * qb, p.v + size_t(row) * p.v_rs + size_t(h0) * p.sk, vb, bar);
      for (int j = 0; j < hg; ++j) {
        cp_async4(&sc[j], p.f + size_t(row) * p.f_rs + size_t(h0 + j) * p.f_hs);
        if (p.i)
          cp_async4(&sc[8 + j], p.i + size_t(row) * p.i_rs + size_t(h0 + j) * p.i_hs);
        else
          sc[8 + j] = 1.0f;
      }
    } else {
      mbar_expect_tx(bar, 0);
    }
    cp_async_arrive(bar);
  }
};

template <int L>
__global__ void __launch_bounds__(kBulkThreads, 2) outer_bulk_kernel(const __grid_constant__ OuterRowsParams p, int hg,
                                                                     int chunk) {
  const Ring r = ring_setup();
  pdl_wait();
  const int groups = p.nh / hg;
  const int items = live_rows(p.at.n_dev, p.at.n_host) * groups;
  const int my = items_of_cta(items, chunk);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  OuterIssue is{p, chunk, hg, groups, uint32_t(hg) * p.sh * p.sk * 4, uint32_t(hg) * p.sh * 4, uint32_t(hg) * p.sk * 4};
  if (warp == 0) {
    if (lane == 0) produce(r, my, p.err, is);
    return;
  }
  const uint32_t sbytes = is.sbytes, qb = is.qb;
  constexpr int RPW = 32 / L;
  const int cw = warp - 1, c4 = lane % L, rsub = lane / L, ctid = threadIdx.x - 32;
  const int wph = kCW / hg;  // warps per head
  const int hh = cw / wph, gw = cw - hh * wph;
  consume(
      r, my, p.err, ctid,
      [&](int k, uint8_t* st) -> bool {
        int row, h0;
        is.item(k, row, h0);
        const float* sc = reinterpret_cast<const float*>(st + kScalarOff);
        float* out = p.out + size_t(row) * p.o_rs + size_t(h0) * p.sk;
        if (sc[kActive] == 0.f) {  // idle row: state untouched, output zero
          for (int i = ctid; i < hg * p.sk; i += kCT) out[i] = 0.f;
          return false;
        }
        float4* S = reinterpret_cast<float4*>(st);
        const float* qs = reinterpret_cast<const float*>(st + kStateMax);
        const float* ks = qs + hg * p.sh;
        const float4* vs = reinterpret_cast<const float4*>(st + kStateMax + 2 * qb);
        const float f = sc[hh], ii = sc[8 + hh];
        const float4 v4 = vs[hh * L + c4];
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int base = gw * RPW; base < p.sh; base += wph * RPW) {  // warp-uniform
          const int i = base + rsub;
          if (i < p.sh) {
            const int e = hh * p.sh + i;
            const float ik = ii * ks[e], qh = qs[e];
            const float4 cur = S[e * L + c4];
            float4 nv;  // f*S + (i*k)*v  (model/kernels.py:143-160)
            nv.x = fmaf(f, cur.x, ik * v4.x);
            nv.y = fmaf(f, cur.y, ik * v4.y);
            nv.z = fmaf(f, cur.z, ik * v4.z);
            nv.w = fmaf(f, cur.w, ik * v4.w);
            S[e * L + c4] = nv;
            acc.x = fmaf(qh, nv.x, acc.x);
            acc.y = fmaf(qh, nv.y, acc.y);
            acc.z = fmaf(qh, nv.z, acc.z);
            acc.w = fmaf(qh, nv.w, acc.w);
          }
        }
#pragma unroll
        for (int o = L; o < 32; o <<= 1) {  // the warp's row groups
          acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
          acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
          acc.z += __shfl_xor_sync(0xffffffffu, acc.z, o);
          acc.w += __shfl_xor_sync(0xffffffffu, acc.w, o);
        }
        // the warps' partial sums, added up in `after` once every warp wrote its own
        if (rsub == 0) r.part[cw * 32 + c4] = acc;
        return true;
      },
      [&](int k, uint8_t* st) {
        int row, h0;
        is.item(k, row, h0);
        const long long slot = *reinterpret_cast<const long long*>(reinterpret_cast<const float*>(st + kScalarOff) + kSlot);
        bulk_store_hint(p.at.state + slot * p.at.row_stride + size_t(h0) * p.sh * p.sk, st, sbytes, l2_evict_first());
      },
      [&](int k, uint8_t*, bool wrote) {
        // past the barrier before the store, so every warp's partials are written;
        // the next item rewrites them only after its first barrier, which every
        // consumer reaches only once done here
        if (!wrote) return;
        int row, h0;
        is.item(k, row, h0);
        float* out = p.out + size_t(row) * p.o_rs + size_t(h0) * p.sk;
        for (int kk = ctid; kk < hg * p.sk; kk += kCT) {  // column kk % sk of head kk / sk
          const int h = kk / p.sk, col = kk - h * p.sk;
          float sum = 0.f;
          for (int w = 0; w < wph; ++w) sum += reinterpret_cast<const float*>(r.part + (h * wph + w) * 32)[col];
          out[kk] = sum;
        }
      });
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int sm_count();
std::atomic<int> g_state_waves{8};

// Grid over `items` (row, head) items. Persistent (waves 0): one CTA per SM, so
// the state kernels of the ensemble step's towers share the SMs with each other
// and with the towers' compute kernels. Alone (waves w > 0): short CTAs of
// `chunk` consecutive items, ~w waves of two CTAs per SM: more copies in flight
// per SM and no tail - 0.96 of measured HBM bandwidth at D2's shapes, against
// 0.86-0.89 persistent; in the ensemble step the persistent grid is faster.
int bulk_grid(long items, const LaunchCfg& ln, int& chunk) {
  const int w = ln.bulk_waves >= 0 ? ln.bulk_waves : g_state_waves.load();
  if (w <= 0) {
    chunk = 0;
    return int(std::min<long>(items, sm_count()));
  }
  const long slots = long(w) * 2 * sm_count();
  chunk = int(std::max<long>(4, (items + slots - 1) / slots));
  return int((items + chunk - 1) / chunk);
}

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Heads per item for the outer kernel: the largest divisor of both nh and kCW
// whose state and operands fit one stage.
int outer_group(const OuterRowsParams& p) {
  const long head = long(p.sh) * p.sk * 4, ops = long(2 * p.sh + p.sk) * 4;
  for (int hg = kCW; hg >= 1; --hg)
    if (p.nh % hg == 0 && kCW % hg == 0 && hg * head <= long(kStateMax) && hg * ops <= long(kScalarOff - kStateMax))
      return hg;
  return 0;
}

template <class K>
void set_bulk_smem(K kernel) {
  B2E_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kBulkSmem)));
}

}  // namespace

void stream_init() {
  int dev = 0;
  B2E_CUDA(cudaGetDevice(&dev));
  static std::once_flag once[64];
  B2E_CHECK(dev >= 0 && dev < 64, kErrInvalid, "device ordinal above 63");
  std::call_once(once[dev], [] {
    set_bulk_smem(ssm_bulk_kernel<32>);
    set_bulk_smem(ssm_bulk_kernel<16>);
    set_bulk_smem(ssm_bulk_kernel<8>);
    set_bulk_smem(outer_bulk_kernel<32>);
    set_bulk_smem(outer_bulk_kernel<16>);
    set_bulk_smem(outer_bulk_kernel<8>);
  });
}

int state_kernel_waves() { return g_state_waves.load(); }
int set_state_kernel_waves(int waves) { return g_state_waves.exchange(std::max(0, waves)); }

bool ssm_cols_bulk_ok(const SsmColsParams& p) {
  return a16(p.at.state) && p.at.row_stride % 4 == 0 && (p.sc == 32 || p.sc == 64 || p.sc == 128) && p.sh > 0 &&
         p.sh % 4 == 0 && p.nh > 0 && long(p.sh) * p.sc * 4 <= long(kStateMax) &&
         long(p.sh) * 4 + long(p.sc) * 8 <= long(kScalarOff - kStateMax) && a16(p.x) && a16(p.b) && a16(p.c) &&
         p.x_rs % 4 == 0 && p.b_rs % 4 == 0 && p.c_rs % 4 == 0 && p.dt && p.decay && p.out;
}

bool outer_rows_bulk_ok(const OuterRowsParams& p) {
  return a16(p.at.state) && p.at.row_stride % 4 == 0 && (p.sk == 32 || p.sk == 64 || p.sk == 128) && p.sh > 0 &&
         p.sh % 4 == 0 && p.nh > 0 && a16(p.q) && a16(p.kv) && a16(p.v) && p.q_rs % 4 == 0 && p.k_rs % 4 == 0 &&
         p.v_rs % 4 == 0 && p.f && p.out && outer_group(p) > 0;
}

void ssm_cols_bulk(const SsmColsParams& p, int rows_max, cudaStream_t s, const LaunchCfg& ln) {
  B2E_CHECK(ssm_cols_bulk_ok(p), kErrInternal, "ssm_cols_bulk: unsupported operands");
  if (rows_max <= 0) return;
  stream_init();
  int chunk = 0;
  const int grid = bulk_grid(long(rows_max) * p.nh, ln, chunk);
  if (p.sc == 128)
    launch_k(ln, ssm_bulk_kernel<32>, dim3(grid), dim3(kBulkThreads), kBulkSmem, s, p, chunk);
  else if (p.sc == 64)
    launch_k(ln, ssm_bulk_kernel<16>, dim3(grid), dim3(kBulkThreads), kBulkSmem, s, p, chunk);
  else
    launch_k(ln, ssm_bulk_kernel<8>, dim3(grid), dim3(kBulkThreads), kBulkSmem, s, p, chunk);
}

void outer_rows_bulk(const OuterRowsParams& p, int rows_max, cudaStream_t s, const LaunchCfg& ln) {
  B2E_CHECK(outer_rows_bulk_ok(p), kErrInternal, "outer_rows_bulk: unsupported operands");
  if (rows_max <= 0) return;
  stream_init();
  const int hg = outer_group(p);
  int chunk = 0;
  const int grid = bulk_grid(long(rows_max) * (p.nh / hg), ln, chunk);
  if (p.sk == 128)
    launch_k(ln, outer_bulk_kernel<32>, dim3(grid), dim3(kBulkThreads), kBulkSmem, s, p, hg, chunk);
  else if (p.sk == 64)
    launch_k(ln, outer_bulk_kernel<16>, dim3(grid), dim3(kBulkThreads), kBulkSmem, s, p, hg, chunk);
  else
    launch_k(ln, outer_bulk_kernel<8>, dim3(grid), dim3(kBulkThreads), kBulkSmem, s, p, hg, chunk);
}

}  // namespace b2e
