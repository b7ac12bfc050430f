// The latency path (see latency.cuh): one kernel per step, one cluster per tower.
//
// Stage plan per tower (H hidden, P proj; every tower starts with IN1, IN2 and
// ends with OUT):
//   IN1   input_up: relu(CastLinear(features))                   -> U1 [P]
//   IN2   input_down                                             -> X  [H]
//   per Block (model/inference_model.py:63-68):
//     layer stages (below), the last one leaves X = X + layer(norm1(X))
//     MLP1  fc1 + ReLU on norm2(X)                               -> Y  [P]
//     MLP2  X + fc2(Y)                                           -> X
//   OUT   output_proj (f32 dot) by the cluster's first CTA.
// Layer stages:
//   Mamba2 (model/mamba2.py:62-168)
//     M1  x|z|b|c projections, dt_proj; conv + SiLU of x, b, c; softplus(dt)
//     M2  ssm update and contraction per p-row; + D*x; * silu(z)  -> A [mi]
//     M3  out_proj(RMSNorm(A)) + X
//   RetNet (model/retnet.py:38-172)
//     R1  q|k|v|g projections; k scaling; rotary; q / sqrt(scales)
//     R2  S update and q.S per column                             -> O [H]
//     R3  out_proj(silu(g) * headRMSNorm(O)) + X
//   Hawk (model/hawk.py:8-95)
//     K1  gate|recurrent projections; conv of the recurrent branch
//     K2  RG-LRU gates (BlockLinear), state update, * gelu(gate)  -> G [H]
//     K3  out_proj(G) + X
//   xLSTM (model/xlstm.py:21-379)
//     A   sLSTM: LayerNorm, conv + SiLU, the eight BlockLinears, the cell
//     B   GroupNorm + skip; LayerNorm; x|gate projections; conv + SiLU;
//         q, k, v BlockLinears
//     C   mLSTM cell per column: gates, stabiliser, n, C, q.C / denominator
//     D   GroupNorm; + skip * conv; * silu(gate); proj_down + skip -> OUT2
//     (MLP1 adds LayerNorm(OUT2) to X before norm2.)
// A stage's outputs are computed for the CTA's slice of the output vector and
// written to the same place in every CTA of the cluster. Every CTA runs every
// stage and every barrier (no CTA leaves early), so the barriers always meet.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstring>

#include "latency.cuh"
#include "mbarrier.cuh"

namespace b2e {
namespace {

namespace cg = cooperative_groups;

constexpr int kCThreads = 256;  // compute warps
constexpr int kPThreads = 64;   // producer warps
constexpr int kThreads = kCThreads + kPThreads;
constexpr int kWarps = kThreads / 32;
// Warps 0-7 run the stages; warps 8-9 (the producer) issue the next stage's
// copies meanwhile. Barriers inside a stage are over the compute warps only
// (named barrier 1); the producer joins them only at the stage's end (the
// cluster barrier). Ten warps cap registers at 168 a thread (a few spill to the
// stack). Measured, one request at D1: 517 us with eight warps and no producer,
// 480 us with seven compute warps and one producer warp, 458 us with eight and
// one, 442 us with eight and two (three or four producer warps: no better).
constexpr int kCWarps = kCThreads / 32;
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kCThreads) : "memory"); }
constexpr float kF32Eps = 1.1920928955078125e-07f;  // nn.RMSNorm(eps=None) in float32

// ----------------------------------------------------------- primitives

#ifdef B2E_LAT_TRACE
// Profiling build only (libb2e_trace.so): %globaltimer stamps around each stage
// of cluster rank 0's thread 0 per tower, read by b2e_lat_trace_read.
constexpr int kTraceStages = 512, kTraceFields = 8;
__device__ unsigned long long g_lat_trace[4][kTraceStages][kTraceFields];
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#endif

__device__ __forceinline__ void cp16(void* dst, const void* src) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp4(void* dst, const void* src) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(d), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_prev() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// rows x row_bytes from src (src_stride bytes apart) into shared memory
// (dst_stride bytes apart), spread over the producer warp's lanes (other
// threads return); asynchronous.
__device__ __forceinline__ void pf2d(void* dst, const void* src, int rows, int row_bytes, long long src_stride,
                                  int dst_stride) {
  if (rows <= 0 || row_bytes <= 0) return;
  const bool v16 = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) == 0 &&
                   (row_bytes & 15) == 0 && (src_stride & 15) == 0 && (dst_stride & 15) == 0;
  const int unit = v16 ? 16 : 4;
  const int per_row = row_bytes / unit;
  const int total = rows * per_row;
  const int pt = int(threadIdx.x) - kCThreads;
  if (pt < 0) return;
  for (int i = pt; i < total; i += kPThreads) {
    const int r = i / per_row, c = i - r * per_row;
    char* d = static_cast<char*>(dst) + size_t(r) * dst_stride + size_t(c) * unit;
    const char* s = static_cast<const char*>(src) + r * src_stride + size_t(c) * unit;
    if (v16)
      cp16(d, s);
    else
      cp4(d, s);
  }
}
// One contiguous segment: no per-chunk row arithmetic.
__device__ __forceinline__ void pf1d(void* dst, const void* src, int bytes) {
  const int pt = int(threadIdx.x) - kCThreads;
  if (bytes <= 0 || pt < 0) return;
  char* d = static_cast<char*>(dst);
  const char* sp = static_cast<const char*>(src);
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | uintptr_t(bytes)) & 15) == 0) {
    for (int i = pt * 16; i < bytes; i += kPThreads * 16) cp16(d + i, sp + i);
  } else {
    for (int i = pt * 4; i < bytes; i += kPThreads * 4) cp4(d + i, sp + i);
  }
}

// A 16-byte aligned bump allocator over one stage buffer; prefetch and compute
// of a stage carve the same sequence, so they agree on every offset.
struct Bump {
  uint8_t* base;
  uint32_t off = 0;
  template <class T>
  __device__ T* take(long long n) {
    off = (off + 15u) & ~15u;
    T* p = reinterpret_cast<T*>(base + off);
    off += uint32_t(n * (long long)sizeof(T));
    return p;
  }
};

template <class WT>
struct WVec;
template <>
struct WVec<float> {
  static constexpr int N = 4;
  __device__ static void load(const float* p, float* o) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
  __device__ static float one(const float* p, int i) { return p[i]; }
  __device__ static float round(float v) { return v; }
};
template <>
struct WVec<__nv_bfloat16> {
  static constexpr int N = 8;
  __device__ static void load(const __nv_bfloat16* p, float* o) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  __device__ static float one(const __nv_bfloat16* p, int i) { return __bfloat162float(p[i]); }
  __device__ static float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <>
struct WVec<__half> {
  static constexpr int N = 8;
  __device__ static void load(const __half* p, float* o) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(h[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
  __device__ static float one(const __half* p, int i) { return __half2float(p[i]); }
  __device__ static float round(float v) { return __half2float(__float2half_rn(v)); }
};

// out[r*ldo + n] = sum_k W[n*ldw + k] * X[r*ldx + k] for n < nrows, r < R.
// W and X in shared memory, W rows 16-byte aligned (ldw elements apart); eight
// lanes per row, four rows per warp at a time.
template <class WT>
__device__ __forceinline__ void gemv(const WT* W, int ldw, int K, int nrows, const float* X, int ldx, int R, float* out,
                                  int ldo) {
  constexpr int V = WVec<WT>::N;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, sub = lane & 7, grp = lane >> 3;
  const int KV = K / V;
  for (int n0 = warp * 4; n0 < nrows; n0 += kCWarps * 4) {
    const int n = n0 + grp;
    float a[kLatMaxRows] = {0.f, 0.f, 0.f, 0.f};
    if (n < nrows) {
      const WT* w = W + size_t(n) * ldw;
      for (int v = sub; v < KV; v += 8) {
        float wf[V];
        WVec<WT>::load(w + v * V, wf);
#pragma unroll
        for (int r = 0; r < kLatMaxRows; ++r) {
          if (r < R) {
            const float* x = X + r * ldx + v * V;
#pragma unroll
            for (int i = 0; i < V; ++i) a[r] = fmaf(wf[i], x[i], a[r]);
          }
        }
      }
      for (int k = KV * V + sub; k < K; k += 8) {
        const float wv = WVec<WT>::one(w, k);
#pragma unroll
        for (int r = 0; r < kLatMaxRows; ++r)
          if (r < R) a[r] = fmaf(wv, X[r * ldx + k], a[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < kLatMaxRows; ++r) {
      a[r] += __shfl_xor_sync(0xffffffffu, a[r], 1);
      a[r] += __shfl_xor_sync(0xffffffffu, a[r], 2);
      a[r] += __shfl_xor_sync(0xffffffffu, a[r], 4);
    }
    if (sub == 0 && n < nrows) {
#pragma unroll
      for (int r = 0; r < kLatMaxRows; ++r)
        if (r < R) out[r * ldo + n] = a[r];
    }
  }
}

// out[r*2 + j] = sum_k W[j*ldw + k] * X[r*ldx + k] for j < 2 rows of a long K,
// with every thread of the CTA (f32 weights). `red` holds kCWarps*8 floats.
__device__ __forceinline__ void dot2_wide(const float* W, int ldw, int K, const float* X, int ldx, int R, float* out,
                                       float* red) {
  float a[2][kLatMaxRows] = {};
  const int K4 = K / 4;
  for (int v = threadIdx.x; v < K4; v += kCThreads) {
    const float4 w0 = *reinterpret_cast<const float4*>(W + 4 * v);
    const float4 w1 = *reinterpret_cast<const float4*>(W + ldw + 4 * v);
#pragma unroll
    for (int r = 0; r < kLatMaxRows; ++r) {
      if (r < R) {
        const float4 x = *reinterpret_cast<const float4*>(X + r * ldx + 4 * v);
        a[0][r] = fmaf(w0.x, x.x, fmaf(w0.y, x.y, fmaf(w0.z, x.z, fmaf(w0.w, x.w, a[0][r]))));
        a[1][r] = fmaf(w1.x, x.x, fmaf(w1.y, x.y, fmaf(w1.z, x.z, fmaf(w1.w, x.w, a[1][r]))));
      }
    }
  }
  for (int k = 4 * K4 + threadIdx.x; k < K; k += kCThreads) {
#pragma unroll
    for (int r = 0; r < kLatMaxRows; ++r) {
      if (r < R) {
        a[0][r] = fmaf(W[k], X[r * ldx + k], a[0][r]);
        a[1][r] = fmaf(W[ldw + k], X[r * ldx + k], a[1][r]);
      }
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int r = 0; r < kLatMaxRows; ++r) {
      const float s = warp_sum(a[j][r]);
      if (lane == 0) red[warp * 8 + j * kLatMaxRows + r] = s;
    }
  csync();
  if (threadIdx.x < 2 * kLatMaxRows) {
    float s = 0.f;
    for (int w = 0; w < kCWarps; ++w) s += red[w * 8 + threadIdx.x];
    const int j = threadIdx.x / kLatMaxRows, r = threadIdx.x % kLatMaxRows;
    if (r < R) out[r * 2 + j] = s;
  }
  csync();
}

// Per row r < R: the sum of f(x[r*ld + i]) over i < n, computed by every warp
// on its own (lanes stride the row, then a shuffle reduction), so no block
// barrier is needed before the result is used. `red` is unused.
template <class F>
__device__ __forceinline__ void row_sums(const float* x, int ld, int n, int R, F f, float* red, float* out) {
  (void)red;
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int r = 0; r < kLatMaxRows; ++r) {
    float a = 0.f;
    if (r < R)
      for (int i = lane; i < n; i += 32) a += f(x[r * ld + i], r);
    out[r] = warp_sum(a);
  }
}

// RMSNorm rows: y = x / sqrt(mean(x^2) + eps) * w (w may be null), over n
// values; y in f32 (yf, may be null) and rounded to the CastLinear type (yl).
template <class WT>
__device__ __forceinline__ void rmsnorm(const float* x, int ld, int n, int R, const float* w, float eps, float* yf, int ldf, float* yl,
                        int ldl, float* red) {
  float ss[kLatMaxRows];
  row_sums(x, ld, n, R, [](float v, int) { return v * v; }, red, ss);
  float inv[kLatMaxRows];
#pragma unroll
  for (int r = 0; r < kLatMaxRows; ++r) inv[r] = 1.0f / sqrtf(ss[r] / float(n) + eps);
  for (int i = threadIdx.x; i < n; i += kCThreads)
#pragma unroll
    for (int r = 0; r < kLatMaxRows; ++r) {
      if (r < R) {
        float y = x[r * ld + i] * inv[r];
        if (w) y *= w[i];
        if (yf) yf[r * ldf + i] = y;
        if (yl) yl[r * ldl + i] = WVec<WT>::round(y);
      }
    }
  csync();
}

// LayerNorm rows (no bias): y = (x - mean) / sqrt(var + eps) * w, handed to
// put(r, i, y), which stores it (and whatever follows from it element-wise).
template <class Put>
__device__ __forceinline__ void layernorm_to(const float* x, int ld, int n, int R, const float* w, float eps, Put put, float* red) {
  float s[kLatMaxRows];
  row_sums(x, ld, n, R, [](float v, int) { return v; }, red, s);
  float mu[kLatMaxRows];
#pragma unroll
  for (int r = 0; r < kLatMaxRows; ++r) mu[r] = s[r] / float(n);
  float q[kLatMaxRows];
  row_sums(x, ld, n, R, [&](float v, int r) { const float d = v - mu[r]; return d * d; }, red, q);
  float inv[kLatMaxRows];
#pragma unroll
  for (int r = 0; r < kLatMaxRows; ++r) inv[r] = 1.0f / sqrtf(q[r] / float(n) + eps);
  for (int i = threadIdx.x; i < n; i += kCThreads)
#pragma unroll
    for (int r = 0; r < kLatMaxRows; ++r)
      if (r < R) put(r, i, (x[r * ld + i] - mu[r]) * inv[r] * w[i]);
  csync();
}

__device__ __forceinline__ void layernorm(const float* x, int ld, int n, int R, const float* w, float eps, float* y, int ldy,
                          float* red) {
  layernorm_to(x, ld, n, R, w, eps, [=](int r, int i, float v) { y[r * ldy + i] = v; }, red);
}

// Mean and 1/sqrt(var + eps) of G groups of gs values per row, one warp per
// (row, group): gm[r*G + g], gr[r*G + g]. Ends with a barrier.
__device__ __forceinline__ void group_stats(const float* x, int ld, int G, int gs, int R, float eps, float* gm, float* gr) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int p = warp; p < R * G; p += kCWarps) {
    const int r = p / G, g = p - r * G;
    const float* v = x + r * ld + g * gs;
    float s = 0.f;
    for (int i = lane; i < gs; i += 32) s += v[i];
    const float mu = warp_sum(s) / float(gs);
    float q = 0.f;
    for (int i = lane; i < gs; i += 32) {
      const float d = v[i] - mu;
      q = fmaf(d, d, q);
    }
    q = warp_sum(q) / float(gs);
    if (lane == 0) {
      gm[p] = mu;
      gr[p] = 1.0f / sqrtf(q + eps);
    }
  }
  csync();
}

// Write src[r*sld + i] (local shared memory, i < cnt) to dst[r*ld + off + i]
// in every CTA of the cluster (dst: this CTA's address of the vector).
__device__ __forceinline__ void bcast(const float* src, int sld, int cnt, int R, float* dst, int ld, int off, int CL) {
  if (cnt <= 0) return;
  cg::cluster_group cluster = cg::this_cluster();
  const bool v4 = (cnt & 3) == 0 && (off & 3) == 0 && (ld & 3) == 0 && (sld & 3) == 0;
  if (v4) {
    const int c4 = cnt >> 2, per = R * c4, total = CL * per;
    for (int i = threadIdx.x; i < total; i += kCThreads) {
      const int peer = i / per, rem = i - peer * per, r = rem / c4, j = rem - r * c4;
      float4* d = reinterpret_cast<float4*>(cluster.map_shared_rank(dst + r * ld + off + 4 * j, peer));
      *d = *reinterpret_cast<const float4*>(src + r * sld + 4 * j);
    }
  } else {
    const int per = R * cnt, total = CL * per;
    for (int i = threadIdx.x; i < total; i += kCThreads) {
      const int peer = i / per, rem = i - peer * per, r = rem / cnt, j = rem - r * cnt;
      *cluster.map_shared_rank(dst + r * ld + off + j, peer) = src[r * sld + j];
    }
  }
}

// CausalConv1d step of one channel (model/modules.py:37-41): the window is the
// tap-major (3, C) state row and x; weights tap-major (4, C).
__device__ __forceinline__ float conv1(const float* w, int C, int c, float bias, float s0, float s1, float s2, float x) {
  float acc = w[c] * s0;
  acc = fmaf(w[C + c], s1, acc);
  acc = fmaf(w[2 * C + c], s2, acc);
  acc = fmaf(w[3 * C + c], x, acc);
  return acc + bias;
}

__device__ __noinline__ float slstm_cell1(float i, float f, float z, float o, float& c, float& n, float& m) {
  // SLSTMCell.forward (model/xlstm.py:247-262)
  const float lfm = m + logsigmoidf_(f);
  const float mn = fmaxf(i, lfm);
  const float og = sigmoidf_(o);
  const float ig = expf(i - mn);
  const float fg = expf(lfm - mn);
  c = fg * c + ig * tanhf(z);
  n = fg * n + ig;
  m = mn;
  return og * c / (n + 1e-6f);
}

__device__ __forceinline__ int rup4(int v) { return (v + 3) & ~3; }

// The CTA's slice [lo, hi) of an N-long output vector.
struct Slice {
  int lo, hi;
  __device__ int n() const { return hi - lo; }
};
__device__ __forceinline__ Slice slice_of(int N, int rank, int CL) {
  const int chunk = rup4((N + CL - 1) / CL);
  const int lo = min(N, rank * chunk);
  return {lo, min(N, lo + chunk)};
}

// ------------------------------------------------------------ the kernel

// Activation vectors in shared memory, [R][len] each (len rounded up to 4).
struct Act {
  float *X, *Xa, *U0, *T, *Y, *U1, *V1, *V2, *HN, *O1, *OUT2, *stg, *red, *gm, *gr, *OW;
  int ldH, ldP, ldT, ld1, ld2;
};

// KIND: the tower's layer kind (its index too); RT: 1 when the step has exactly
// one row (every row loop folds away), 0 for up to kLatMaxRows rows.
template <class WT, int KIND, int RT>
struct Tower {
  const LatModel& M;
  const LatTower* T;       // this tower's descriptor (a shared-memory copy in the step kernel)
  const LatBlock* blocks;  // its blocks (likewise)
  long long* slot;         // the step's state slots (shared memory)
  const LatIO& io;
  int fpad, F, depth;
  static constexpr int kind = KIND;
  int rank, CL, R, RM, H, P, mi, nh_m, hs_m, bc, nh, hs_r, nbl, bs, hs_x, nh_x;  // RM: rows the carve holds
  Act a;
  bool dry = false;  // carve only (the planning pass sizes the buffers this way)
  uint32_t act_used = 0;
  __device__ void P2(void* dst, const void* src, int rows, int row_bytes, long long src_stride, int dst_stride) {
    if (!dry) pf2d(dst, src, rows, row_bytes, src_stride, dst_stride);
  }
  __device__ void P1(void* dst, const void* src, int bytes) {
    if (!dry) pf1d(dst, src, bytes);
  }

  // Carves the shared memory at act_base: descriptors and slots first, then the
  // activation vectors. `t` is the tower's descriptor until load_desc() points
  // T and blocks at the shared-memory copies.
  __device__ Tower(const LatModel& m, const LatTower& t, const LatIO& i, int rk, int cl, uint8_t* act_base)
      : M(m), T(&t), blocks(t.blocks), io(i) {
    rank = rk; CL = cl; R = RT ? RT : i.n; RM = m.rmax;
    fpad = m.fpad; F = m.F; depth = m.depth;
    H = m.H; P = m.P;
    mi = 2 * H; nh_m = mi / m.m_hs; hs_m = m.m_hs; bc = m.m_bc;
    nh = m.heads; hs_r = H / nh;
    nbl = nh / 2; bs = H / nbl;
    nh_x = nh; hs_x = mi / nh;
    Bump b{act_base};
    dT = b.take<LatTower>(1);
    dB = b.take<LatBlock>(depth);
    slot = b.take<long long>(kLatMaxRows);
    a.ldH = rup4(H); a.ldP = rup4(P); a.ldT = rup4(max(max(H, mi), max(P, m.fpad)));
    a.ld1 = rup4(len1()); a.ld2 = rup4(len2());
    a.X = b.take<float>(RM * a.ldH);
    a.Xa = b.take<float>(RM * a.ldH);
    a.U0 = b.take<float>(RM * a.ldH);
    a.HN = b.take<float>(RM * a.ldH);
    a.O1 = b.take<float>(RM * a.ldH);
    a.OUT2 = b.take<float>(RM * a.ldH);
    a.T = b.take<float>(RM * a.ldT);
    a.Y = b.take<float>(RM * a.ldP);
    a.U1 = a.Y;  // input_up's output is dead once input_down has read it
    a.V1 = b.take<float>(RM * a.ld1);
    a.V2 = b.take<float>(RM * a.ld2);
    a.stg = b.take<float>(RM * stg_len());
    a.red = b.take<float>(kCWarps * 8);
    a.gm = b.take<float>(RM * 64);
    a.gr = b.take<float>(RM * 64);
    a.OW = b.take<float>(a.ldH);
    act_used = (b.off + 127u) & ~127u;
  }
  // the per-tower broadcast vectors: V1 = the first layer stage's outputs, V2 the second's
  __device__ int len1() const {
    switch (kind) {
      case kMamba2: return 2 * mi + 2 * bc + nh_m;  // xs | z | bs | cs | dt
      case kRetNet: return 4 * H;                   // qs | kr | v | g
      case kHawk: return 2 * H;                     // gate | xc
      default: return 5 * mi;                       // xc | xg | q | k | v
    }
  }
  __device__ int len2() const {
    switch (kind) {
      case kMamba2: return mi;  // A
      case kRetNet: return H;   // O
      case kHawk: return H;     // G
      default: return mi;       // O (mLSTM cell out)
    }
  }
  // staging floats per row: the largest output slice any stage stages (RetNet's
  // rotary keeps two copies, the mLSTM stages keep q/k/v or k, n beside it)
  __device__ int chunk(int N) const { return rup4((N + CL - 1) / CL); }
  __device__ int stg_len() const {
    int v = max(max(chunk(P), chunk(H)), chunk(len1()));
    v = max(v, 2 * chunk(4 * H));
    v = max(v, 5 * chunk(2 * mi));
    v = max(v, 5 * chunk(H));
    v = max(v, 2 * hs_x + 4 + chunk(mi));
    return rup4(v + 16);
  }
  __device__ int per_block() const { return kind == kXLSTM ? 6 : 5; }
  __device__ int nstages() const { return 2 + depth * per_block(); }

  LatTower* dT = nullptr;
  LatBlock* dB = nullptr;
  // Copy the tower's descriptors and the step's slots into shared memory (every
  // thread takes part; ends with a barrier), so no stage chases pointers in HBM.
  __device__ void load_desc() {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(T);
    uint32_t* dst = reinterpret_cast<uint32_t*>(dT);
    for (int k = threadIdx.x; k < int(sizeof(LatTower) / 4); k += kThreads) dst[k] = src[k];
    const uint32_t* bs_ = reinterpret_cast<const uint32_t*>(blocks);
    uint32_t* bd = reinterpret_cast<uint32_t*>(dB);
    for (int k = threadIdx.x; k < int(depth * sizeof(LatBlock) / 4); k += kThreads) bd[k] = bs_[k];
    if (threadIdx.x < kLatMaxRows) slot[threadIdx.x] = threadIdx.x < R ? io.slots[threadIdx.x] : 0;
    __syncthreads();
    T = dT;
    blocks = dB;
  }

  // Small per-stage vectors of the prologue (norm weights, gate biases, ...),
  // first in each stage buffer so no stage waits on an L2 round trip for them.
  struct SV {
    const float* p[4];
  };
  __device__ SV small_vecs(int j, const LatBlock& B, Bump& b, bool issue) {
    SV v{};
    auto add = [&](int i, const void* src, int n) {
      float* d = b.take<float>(n);
      if (issue) P1(d, src, n * 4);
      v.p[i] = d;
    };
    const LatLayer& L = B.L;
    if (j == per_block() - 2) {
      add(0, B.n2, H);
      if (kind == kXLSTM) add(1, L.w[20], H);
      return v;
    }
    if (j == per_block() - 1) return v;
    if (j == 0) add(0, B.n1, H);
    switch (kind) {
      case kMamba2:
        if (j == 0) add(1, L.w[2], nh_m);
        if (j == 1) { add(1, L.w[9], nh_m); add(2, L.w[10], nh_m); }
        if (j == 2) add(1, L.w[11], mi);
        break;
      case kRetNet:
        if (j == 0) { add(1, L.w[3], hs_r); add(2, L.w[2], nh); }
        if (j == 1) add(2, L.w[2], nh);
        break;
      case kHawk:
        break;
      default:
        if (j == 0) add(1, L.w[0], H);
        if (j == 1) { add(1, L.w[5], H); add(2, L.w[6], H); add(3, L.w[8], H); }
        if (j == 2) add(1, L.w[16], 2 * nh_x);
        if (j == 3) { add(1, L.w[17], mi); add(2, L.w[18], mi); add(3, L.w[7], mi); }
        break;
    }
    return v;
  }

  // =============================================================== prefetch
  __device__ uint32_t prefetch(int s, uint8_t* buf) {
    Bump b{buf};
    prefetch_into(s, b);
    return b.off;
  }
  __device__ void prefetch_into(int s, Bump& b) {
    if (s == 0) {
      const Slice sl = slice_of(P, rank, CL);
      P2(b.take<WT>(sl.n() * fpadw()), static_cast<const WT*>(T->upw) + size_t(sl.lo) * fpad, sl.n(),
           fpad * sizeof(WT), fpad * sizeof(WT), fpadw() * sizeof(WT));
      P1(b.take<WT>(sl.n()), static_cast<const WT*>(T->upb) + sl.lo, sl.n() * sizeof(WT));
      return;
    }
    if (s == 1) {
      const Slice sl = slice_of(H, rank, CL);
      P1(b.take<WT>(size_t(sl.n()) * P), static_cast<const WT*>(T->dnw) + size_t(sl.lo) * P, sl.n() * P * sizeof(WT));
      P1(b.take<WT>(sl.n()), static_cast<const WT*>(T->dnb) + sl.lo, sl.n() * sizeof(WT));
      return;
    }
    const int blk = (s - 2) / per_block(), j = (s - 2) % per_block();
    const LatBlock& B = blocks[blk];
    small_vecs(j, B, b, true);
    if (j == per_block() - 2) {  // MLP1: fc1
      const Slice sl = slice_of(P, rank, CL);
      P1(b.take<WT>(size_t(sl.n()) * H), static_cast<const WT*>(B.f1w) + size_t(sl.lo) * H, sl.n() * H * sizeof(WT));
      P1(b.take<WT>(sl.n()), static_cast<const WT*>(B.f1b) + sl.lo, sl.n() * sizeof(WT));
      return;
    }
    if (j == per_block() - 1) {  // MLP2: fc2
      const Slice sl = slice_of(H, rank, CL);
      P1(b.take<WT>(size_t(sl.n()) * P), static_cast<const WT*>(B.f2w) + size_t(sl.lo) * P, sl.n() * P * sizeof(WT));
      P1(b.take<WT>(sl.n()), static_cast<const WT*>(B.f2b) + sl.lo, sl.n() * sizeof(WT));
      return;
    }
    switch (kind) {
      case kMamba2: return pf_mamba(j, B.L, b);
      case kRetNet: return pf_retnet(j, B.L, b);
      case kHawk: return pf_hawk(j, B.L, b);
      default: return pf_xlstm(j, B.L, b);
    }
  }
  __device__ int fpadw() const { return (fpad * int(sizeof(WT)) + 15) / 16 * 16 / int(sizeof(WT)); }

  // state rows of a (3, C) conv leaf for channels [lo, hi): three segments per row
  __device__ float* pf_conv(Bump& b, float* base, long long stride, int C, int lo, int hi) {
    float* d = b.take<float>(RM * 3 * (hi - lo));
    for (int r = 0; r < R; ++r)
      P2(d + r * 3 * (hi - lo), base + slot[r] * stride + lo, 3, (hi - lo) * 4, C * 4ll, (hi - lo) * 4);
    return d;
  }
  __device__ float* pf_rows(Bump& b, const float* base, long long stride, int off, int cnt) {
    float* d = b.take<float>(RM * cnt);
    for (int r = 0; r < R; ++r) P1(d + r * cnt, base + slot[r] * stride + off, cnt * 4);
    return d;
  }

  // ------------------------------------------------------------- Mamba2
  // w: 0 w1 [x|z|b|c][H] (lp), 1 dt_proj W [nh][H], 2 dt bias, 3 x conv W (4, mi), 4 x conv b,
  // 5 b conv W, 6 b conv b, 7 c conv W, 8 c conv b, 9 a, 10 d, 11 norm W [mi], 12 out_proj [H][mi] (lp)
  // st: 0 x conv (3, mi), 1 b conv (3, bc), 2 c conv (3, bc), 3 ssm (nh, hs, bc)
  struct MambaM1 {
    Slice sl;
    int xl, xh, zl, zh, bl, bh, cl, ch, dl, dh;  // sub-ranges by output kind, in each kind's own index
  };
  __device__ MambaM1 m1_ranges() const {
    MambaM1 q;
    q.sl = slice_of(len1(), rank, CL);
    auto clip = [&](int base, int len, int& l, int& h) {
      l = max(q.sl.lo, base) - base;
      h = min(q.sl.hi, base + len) - base;
      if (h < l) h = l = 0;
    };
    clip(0, mi, q.xl, q.xh);
    clip(mi, mi, q.zl, q.zh);
    clip(2 * mi, bc, q.bl, q.bh);
    clip(2 * mi + bc, bc, q.cl, q.ch);
    clip(2 * mi + 2 * bc, nh_m, q.dl, q.dh);
    return q;
  }
  __device__ void pf_mamba(int j, const LatLayer& L, Bump& b) {
    if (j == 0) {
      const MambaM1 q = m1_ranges();
      const int nl = min(q.sl.hi, 2 * mi + 2 * bc) - min(q.sl.lo, 2 * mi + 2 * bc);
      P1(b.take<WT>(size_t(nl) * H), static_cast<const WT*>(L.w[0]) + size_t(q.sl.lo) * H, nl * H * sizeof(WT));
      P1(b.take<float>(size_t(q.dh - q.dl) * H), static_cast<const float*>(L.w[1]) + size_t(q.dl) * H,
           (q.dh - q.dl) * H * 4);
      const int cc[3][2] = {{q.xl, q.xh}, {q.bl, q.bh}, {q.cl, q.ch}};
      const int CC[3] = {mi, bc, bc};
      for (int t = 0; t < 3; ++t) {
        const int lo = cc[t][0], hi = cc[t][1];
        P2(b.take<float>(4 * (hi - lo)), static_cast<const float*>(L.w[3 + 2 * t]) + lo, 4, (hi - lo) * 4,
             CC[t] * 4ll, (hi - lo) * 4);
        P1(b.take<float>(hi - lo), static_cast<const float*>(L.w[4 + 2 * t]) + lo, (hi - lo) * 4);
        pf_conv(b, L.st[t], L.ss[t], CC[t], lo, hi);
      }
      return;
    }
    if (j == 1) {
      const Slice sl = slice_of(mi, rank, CL);
      pf_rows(b, L.st[3], L.ss[3], sl.lo * bc, sl.n() * bc);
      return;
    }
    const Slice sl = slice_of(H, rank, CL);
    P1(b.take<WT>(size_t(sl.n()) * mi), static_cast<const WT*>(L.w[12]) + size_t(sl.lo) * mi, sl.n() * mi * sizeof(WT));
  }

  __device__ void run_mamba(int j, const LatLayer& L, Bump& b, const SV& sv) {
    if (j == 0) {
      const MambaM1 q = m1_ranges();
      rmsnorm<WT>(a.X, a.ldH, H, R, sv.p[0], kF32Eps, a.U0, a.ldH, a.T, a.ldT, a.red);  // norm1, then x.to(lp)
      const int nl = min(q.sl.hi, 2 * mi + 2 * bc) - min(q.sl.lo, 2 * mi + 2 * bc);
      const WT* w1 = b.take<WT>(size_t(nl) * H);
      const float* dtw = b.take<float>(size_t(q.dh - q.dl) * H);
      const int ld = rup4(q.sl.n());
      gemv<WT>(w1, H, H, nl, a.T, a.ldT, R, a.stg, ld);
      gemv<float>(dtw, H, H, q.dh - q.dl, a.U0, a.ldH, R, a.stg + nl, ld);  // dt_proj keeps fp32 (example_model.py:106)
      csync();
      const int cc[3][2] = {{q.xl, q.xh}, {q.bl, q.bh}, {q.cl, q.ch}};
      const int base[3] = {0, 2 * mi, 2 * mi + bc};
      const int CC[3] = {mi, bc, bc};
      const float* cw[3];
      const float* cb[3];
      const float* cs[3];
      for (int t = 0; t < 3; ++t) {
        const int n = cc[t][1] - cc[t][0];
        cw[t] = b.take<float>(4 * n);
        cb[t] = b.take<float>(n);
        cs[t] = b.take<float>(RM * 3 * n);
      }
      const float* dtb = sv.p[1];
      for (int i = threadIdx.x; i < q.sl.n() * R; i += kCThreads) {
        const int r = i / q.sl.n(), e = i - r * q.sl.n(), idx = q.sl.lo + e;
        float& v = a.stg[r * ld + e];
        if (idx < 2 * mi + 2 * bc) {
          v = WVec<WT>::round(v);  // CastLinear output
          // x rows [0, mi) and the b, c rows go through their convs; z rows [mi, 2mi) do not
          const int t = idx < mi ? 0 : idx < 2 * mi ? -1 : idx < 2 * mi + bc ? 1 : 2;
          if (t >= 0) {
            const int c = idx - base[t], n = cc[t][1] - cc[t][0], k = c - cc[t][0];
            const float* st = cs[t] + r * 3 * n;
            const float y = conv1(cw[t], n, k, cb[t][k], st[k], st[n + k], st[2 * n + k], v);
            float* g = L.st[t] + slot[r] * L.ss[t];  // window shifts by one (model/modules.py:41)
            g[c] = st[n + k];
            g[CC[t] + c] = st[2 * n + k];
            g[2 * CC[t] + c] = v;
            v = siluf_(y);  // mamba2.py:89-91
          }
        } else {
          const int h = idx - (2 * mi + 2 * bc);
          v = softplusf_(v + dtb[h]);  // mamba2.py:96
        }
      }
      csync();
      bcast(a.stg, ld, q.sl.n(), R, a.V1, a.ld1, q.sl.lo, CL);
      return;
    }
    if (j == 1) {
      // ssm update per p-row (mamba2.py:99-117): h = decay*h + (dt*b)*x; y = c.h + d*x; y * silu(z)
      const Slice sl = slice_of(mi, rank, CL);
      float* ssm = b.take<float>(RM * sl.n() * bc);
      const float* a_ = sv.p[1];
      const float* d_ = sv.p[2];
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
      for (int pr = warp; pr < sl.n() * R; pr += kCWarps) {
        const int r = pr / sl.n(), p = sl.lo + (pr - r * sl.n()), n = p / hs_m;
        const float* v = a.V1 + r * a.ld1;
        const float x = v[p], dt = v[2 * mi + 2 * bc + n];
        const float dc = expf(a_[n] * dt);  // decay = exp(a * dt) (mamba2.py:97)
        float* h = ssm + (size_t(r) * sl.n() + (p - sl.lo)) * bc;
        float* g = L.st[3] + slot[r] * L.ss[3] + size_t(p) * bc;
        float y = 0.f;
        for (int c = lane; c < bc; c += 32) {
          const float bv = v[2 * mi + c], cv = v[2 * mi + bc + c];
          const float hn = dc * h[c] + (dt * bv) * x;
          g[c] = hn;
          y = fmaf(cv, hn, y);
        }
        y = warp_sum(y);
        if (lane == 0) {
          y = y + d_[n] * x;
          a.stg[r * rup4(sl.n()) + (p - sl.lo)] = y * siluf_(v[mi + p]);  // y * silu(z) (mamba2.py:160)
        }
      }
      csync();
      bcast(a.stg, rup4(sl.n()), sl.n(), R, a.V2, a.ld2, sl.lo, CL);
      return;
    }
    // M3: out_proj(RMSNorm(A)) + X (mamba2.py:161-165)
    rmsnorm<WT>(a.V2, a.ld2, mi, R, sv.p[1], 1e-5f, nullptr, 0, a.T, a.ldT, a.red);
    const Slice sl = slice_of(H, rank, CL);
    const WT* w = b.take<WT>(size_t(sl.n()) * mi);
    residual_out(w, mi, sl, nullptr);
  }

  // X[n] += round(W x) for the CTA's slice (x = a.T, K wide), broadcast X.
  __device__ void residual_out(const WT* w, int K, Slice sl, const WT* bias) {
    const int ld = rup4(sl.n());
    gemv<WT>(w, K, K, sl.n(), a.T, a.ldT, R, a.stg, ld);
    csync();
    for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
      const int r = i / sl.n(), e = i - r * sl.n();
      float v = a.stg[r * ld + e];
      if (bias) v += WVec<WT>::one(bias, e);
      a.stg[r * ld + e] = a.X[r * a.ldH + sl.lo + e] + WVec<WT>::round(v);
    }
    csync();
    bcast(a.stg, ld, sl.n(), R, a.X, a.ldH, sl.lo, CL);
  }

  // ------------------------------------------------------------- RetNet
  // w: 0 w1 [q|k|v|g][H] (lp), 1 out_proj [H][H] (lp), 2 decay [nh], 3 angle [hs]
  // st: 0 pos (int), 1 scales [nh], 2 S (nh, hs, hs)
  __device__ void pf_retnet(int j, const LatLayer& L, Bump& b) {
    if (j == 0) {
      const Slice sl = slice_of(4 * H, rank, CL);
      P1(b.take<WT>(size_t(sl.n()) * H), static_cast<const WT*>(L.w[0]) + size_t(sl.lo) * H, sl.n() * H * sizeof(WT));
      pf_rows(b, L.st[1], L.ss[1], 0, nh);
      pf_rows(b, L.st[0], L.ss[0], 0, 1);  // position counters (int32, copied as words)
      return;
    }
    if (j == 1) {
      const Slice sl = slice_of(H, rank, CL);
      float* d = b.take<float>(RM * hs_r * sl.n());
      for (int r = 0; r < R; ++r) {
        // columns [lo, hi) may span heads: one strided copy per head touched
        for (int e = sl.lo; e < sl.hi;) {
          const int n = e / hs_r, kk = e - n * hs_r, cnt = min(sl.hi - e, hs_r - kk);
          P2(d + size_t(r) * hs_r * sl.n() + (e - sl.lo), L.st[2] + slot[r] * L.ss[2] + size_t(n) * hs_r * hs_r + kk,
               hs_r, cnt * 4, hs_r * 4ll, sl.n() * 4);
          e += cnt;
        }
      }
      return;
    }
    const Slice sl = slice_of(H, rank, CL);
    P1(b.take<WT>(size_t(sl.n()) * H), static_cast<const WT*>(L.w[1]) + size_t(sl.lo) * H, sl.n() * H * sizeof(WT));
  }

  __device__ void run_retnet(int j, const LatLayer& L, Bump& b, const SV& sv) {
    if (j == 0) {
      rmsnorm<WT>(a.X, a.ldH, H, R, sv.p[0], kF32Eps, nullptr, 0, a.T, a.ldT, a.red);
      const Slice sl = slice_of(4 * H, rank, CL);
      const WT* w = b.take<WT>(size_t(sl.n()) * H);
      const float* sc = b.take<float>(RM * nh);
      const int* posv = reinterpret_cast<const int*>(b.take<float>(RM));
      const int ld = rup4(sl.n());
      gemv<WT>(w, H, H, sl.n(), a.T, a.ldT, R, a.stg, ld);
      csync();
      for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
        const int r = i / sl.n(), e = i - r * sl.n();
        a.stg[r * ld + e] = WVec<WT>::round(a.stg[r * ld + e]);  // CastLinear outputs q, k, v, g
      }
      csync();
      const float* angle = sv.p[1];
      const float* decay = sv.p[2];
      const float scaling = powf(float(hs_r), -0.5f);
      // rotary and scaling into a second half of the staging area (pairs read both lanes' inputs)
      float* out = a.stg + R * ld;
      for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
        const int r = i / sl.n(), e = i - r * sl.n(), idx = sl.lo + e;
        float v = a.stg[r * ld + e];
        if (idx < 2 * H) {
          const int part = idx / H, ee = idx - part * H, n = ee / hs_r, jj = ee - n * hs_r;
          const int mate = (jj & 1) ? e - 1 : e + 1;  // same slice: slices are 4-aligned, heads even
          const float fpos = float(posv[r]);  // int32 counter promoted to float32 (retnet.py:78)
          const float arg = fpos * angle[jj];
          const float sn = sinf(arg), co = cosf(arg);
          float x = v, xm = a.stg[r * ld + mate];
          if (part == 1) {  // k *= hs^-1/2 (retnet.py:71)
            x = x * scaling;
            xm = xm * scaling;
          }
          const float rot = (jj & 1) ? xm : -xm;  // rotate_every_two (retnet.py:9-13)
          v = x * co + rot * sn;
          if (part == 0) {
            const float ns = sc[r * nh + n] * decay[n] + 1.0f;  // retnet.py:93
            v = v * (1.0f / sqrtf(ns));
          }
        }
        out[r * ld + e] = v;
      }
      csync();
      // the CTA holding a head's first q element advances that head's scale;
      // the first CTA advances the position (retnet.py:93, 172)
      for (int i = threadIdx.x; i < nh * R; i += kCThreads) {
        const int r = i / nh, n = i - r * nh;
        if (n * hs_r >= sl.lo && n * hs_r < sl.hi) L.st[1][slot[r] * L.ss[1] + n] = sc[r * nh + n] * decay[n] + 1.0f;
      }
      if (rank == 0 && threadIdx.x < R)
        reinterpret_cast<int*>(L.st[0])[slot[threadIdx.x] * L.ss[0]] = posv[threadIdx.x] + 1;
      bcast(out, ld, sl.n(), R, a.V1, a.ld1, sl.lo, CL);
      return;
    }
    if (j == 1) {
      // per column e = n*hs + kk (retnet.py:129-140): S = decay*S + k x v; o = q.S
      const Slice sl = slice_of(H, rank, CL);
      float* S = b.take<float>(RM * hs_r * sl.n());
      const float* decay = sv.p[2];
      const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, ld = rup4(sl.n());
      for (int pc = warp; pc < sl.n() * R; pc += kCWarps) {
        const int r = pc / sl.n(), c = pc - r * sl.n(), e = sl.lo + c, n = e / hs_r, kk = e - n * hs_r;
        const float* v1 = a.V1 + r * a.ld1;
        const float ve = v1[2 * H + e], g = decay[n];
        float* g_row = L.st[2] + slot[r] * L.ss[2] + size_t(n) * hs_r * hs_r + kk;
        float o = 0.f;
        for (int h = lane; h < hs_r; h += 32) {
          const float sv = S[(size_t(r) * hs_r + h) * sl.n() + c];
          const float sn = sv * g + v1[H + n * hs_r + h] * ve;
          g_row[size_t(h) * hs_r] = sn;
          o = fmaf(v1[n * hs_r + h], sn, o);
        }
        o = warp_sum(o);
        if (lane == 0) a.stg[r * ld + c] = o;
      }
      csync();
      bcast(a.stg, ld, sl.n(), R, a.V2, a.ld2, sl.lo, CL);
      return;
    }
    // R3: silu(g) * headRMSNorm(O) -> out_proj + X (retnet.py:168-170)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int p = warp; p < R * nh; p += kCWarps) {
      const int r = p / nh, n = p - r * nh;
      const float* o = a.V2 + r * a.ld2 + n * hs_r;
      float ss = 0.f;
      for (int i = lane; i < hs_r; i += 32) ss = fmaf(o[i], o[i], ss);
      ss = warp_sum(ss);
      if (lane == 0) a.gr[p] = 1.0f / sqrtf(ss / float(hs_r) + 1e-6f);
    }
    csync();
    for (int i = threadIdx.x; i < H * R; i += kCThreads) {
      const int r = i / H, e = i - r * H;
      const float g = a.V1[r * a.ld1 + 3 * H + e];
      a.T[r * a.ldT + e] = WVec<WT>::round(siluf_(g) * (a.V2[r * a.ld2 + e] * a.gr[r * nh + e / hs_r]));
    }
    csync();
    const Slice sl = slice_of(H, rank, CL);
    residual_out(b.take<WT>(size_t(sl.n()) * H), H, sl, nullptr);
  }

  // --------------------------------------------------------------- Hawk
  // w: 0 w1 [gate|rec][H] (lp), 1 conv W (4, H), 2 conv b, 3 a [H], 4 gate W [2][4][bs][bs], 5 out_proj (lp)
  // st: 0 conv (3, H), 1 h [H]
  __device__ void pf_hawk(int j, const LatLayer& L, Bump& b) {
    if (j == 0) {
      const Slice sl = slice_of(2 * H, rank, CL);
      P1(b.take<WT>(size_t(sl.n()) * H), static_cast<const WT*>(L.w[0]) + size_t(sl.lo) * H, sl.n() * H * sizeof(WT));
      const int lo = max(sl.lo, H) - H, hi = max(sl.hi, H) - H;  // recurrent-branch channels
      P2(b.take<float>(4 * (hi - lo)), static_cast<const float*>(L.w[1]) + lo, 4, (hi - lo) * 4, H * 4ll,
           (hi - lo) * 4);
      P1(b.take<float>(hi - lo), static_cast<const float*>(L.w[2]) + lo, (hi - lo) * 4);
      pf_conv(b, L.st[0], L.ss[0], H, lo, hi);
      return;
    }
    if (j == 1) {
      const Slice sl = slice_of(H, rank, CL);
      const int hb = H / 4;  // RG-LRU blocks (hawk.py:16)
      float* gw = b.take<float>(2 * sl.n() * hb);
      for (int s = 0; s < 2; ++s)
        for (int c = sl.lo; c < sl.hi;) {
          const int jb = c / hb, e = c - jb * hb, cnt = min(sl.hi - c, hb - e);
          P1(gw + (size_t(s) * sl.n() + (c - sl.lo)) * hb,
               static_cast<const float*>(L.w[4]) + ((size_t(s) * 4 + jb) * hb + e) * hb, cnt * hb * 4);
          c += cnt;
        }
      P1(b.take<float>(sl.n()), static_cast<const float*>(L.w[3]) + sl.lo, sl.n() * 4);
      pf_rows(b, L.st[1], L.ss[1], sl.lo, sl.n());
      return;
    }
    const Slice sl = slice_of(H, rank, CL);
    P1(b.take<WT>(size_t(sl.n()) * H), static_cast<const WT*>(L.w[5]) + size_t(sl.lo) * H, sl.n() * H * sizeof(WT));
  }

  __device__ void run_hawk(int j, const LatLayer& L, Bump& b, const SV& sv) {
    if (j == 0) {
      rmsnorm<WT>(a.X, a.ldH, H, R, sv.p[0], kF32Eps, nullptr, 0, a.T, a.ldT, a.red);
      const Slice sl = slice_of(2 * H, rank, CL);
      const WT* w = b.take<WT>(size_t(sl.n()) * H);
      const int lo = max(sl.lo, H) - H, hi = max(sl.hi, H) - H, n = hi - lo;
      const float* cw = b.take<float>(4 * n);
      const float* cb = b.take<float>(n);
      const float* cs = b.take<float>(RM * 3 * n);
      const int ld = rup4(sl.n());
      gemv<WT>(w, H, H, sl.n(), a.T, a.ldT, R, a.stg, ld);
      csync();
      for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
        const int r = i / sl.n(), e = i - r * sl.n(), idx = sl.lo + e;
        float v = WVec<WT>::round(a.stg[r * ld + e]);
        if (idx >= H) {  // recurrent branch -> conv (hawk.py:79-80)
          const int c = idx - H, k = c - lo;
          const float* st = cs + r * 3 * n;
          const float y = conv1(cw, n, k, cb[k], st[k], st[n + k], st[2 * n + k], v);
          float* g = L.st[0] + slot[r] * L.ss[0];
          g[c] = st[n + k];
          g[H + c] = st[2 * n + k];
          g[2 * H + c] = v;
          v = y;
        }
        a.stg[r * ld + e] = v;
      }
      csync();
      bcast(a.stg, ld, sl.n(), R, a.V1, a.ld1, sl.lo, CL);
      return;
    }
    if (j == 1) {
      // RG-LRU (hawk.py:27-38) and the gate (hawk.py:77, 83)
      const Slice sl = slice_of(H, rank, CL);
      const int hb = H / 4;
      const float* gw = b.take<float>(2 * sl.n() * hb);
      const float* av = b.take<float>(sl.n());
      const float* hs = b.take<float>(RM * sl.n());
      const int ld = rup4(sl.n()), lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
      for (int pc = warp; pc < sl.n() * R; pc += kCWarps) {
        const int r = pc / sl.n(), c = pc - r * sl.n(), ch = sl.lo + c, jb = ch / hb;
        const float* xc = a.V1 + r * a.ld1 + H + jb * hb;
        float gi = 0.f, gr = 0.f;
        for (int k = lane; k < hb; k += 32) {
          gi = fmaf(gw[size_t(c) * hb + k], xc[k], gi);
          gr = fmaf(gw[(size_t(sl.n()) + c) * hb + k], xc[k], gr);
        }
        gi = warp_sum(gi);
        gr = warp_sum(gr);
        if (lane == 0) {
          const float it = sigmoidf_(gi), rt = sigmoidf_(gr);
          const float at = powf(av[c], 8.0f * rt);
          const float mult = sqrtf(1.0f - at * at);
          const float x = a.V1[r * a.ld1 + H + ch];
          const float hn = hs[r * sl.n() + c] * at + mult * (it * x);
          L.st[1][slot[r] * L.ss[1] + ch] = hn;
          a.stg[r * ld + c] = geluf_(a.V1[r * a.ld1 + ch]) * hn;
        }
      }
      csync();
      bcast(a.stg, ld, sl.n(), R, a.V2, a.ld2, sl.lo, CL);
      return;
    }
    for (int i = threadIdx.x; i < H * R; i += kCThreads) {
      const int r = i / H, e = i - r * H;
      a.T[r * a.ldT + e] = WVec<WT>::round(a.V2[r * a.ld2 + e]);
    }
    csync();
    const Slice sl = slice_of(H, rank, CL);
    residual_out(b.take<WT>(size_t(sl.n()) * H), H, sl, nullptr);
  }

  // -------------------------------------------------------------- xLSTM
  // w: 0 sLSTM LN W, 1 sLSTM conv W (4, H), 2 conv b, 3 gate W [4][nbl][bs][2bs], 4 gate bias [4][H],
  // 5 GN W, 6 GN b, 7 learnable_skip [mi], 8 mLSTM LN W, 9 x|gate proj [2mi][H] (lp), 10 q, 11 k,
  // 12 v BlockLinear [mi/4][4][4], 13 mLSTM conv W (4, mi), 14 conv b, 15 i|f gate W [2nh][3mi],
  // 16 i|f gate b, 17 outnorm W, 18 outnorm b, 19 proj_down [H][mi] (lp), 20 final LN W
  // st: 0 sLSTM conv (3, H), 1 h, 2 c, 3 n, 4 m, 5 mLSTM conv (3, mi), 6 C (nh, hs, hs), 7 n (nh, hs), 8 m (nh)
  __device__ void pf_xlstm(int j, const LatLayer& L, Bump& b) {
    if (j == 0) {
      const Slice sl = slice_of(H, rank, CL);
      if (sl.n() == 0) return;  // no channels here: no head block to read
      const int jb = sl.lo / bs, b0 = jb * bs;
      for (int g = 0; g < 4; ++g)
        P1(b.take<float>(size_t(sl.n()) * 2 * bs),
             static_cast<const float*>(L.w[3]) + ((size_t(g) * nbl + jb) * bs + (sl.lo - b0)) * 2 * bs,
             sl.n() * 2 * bs * 4);
      float* bias = b.take<float>(4 * sl.n());
      for (int g = 0; g < 4; ++g) P1(bias + g * sl.n(), static_cast<const float*>(L.w[4]) + g * H + sl.lo, sl.n() * 4);
      P2(b.take<float>(4 * bs), static_cast<const float*>(L.w[1]) + b0, 4, bs * 4, H * 4ll, bs * 4);
      P1(b.take<float>(bs), static_cast<const float*>(L.w[2]) + b0, bs * 4);
      pf_conv(b, L.st[0], L.ss[0], H, b0, b0 + bs);
      pf_rows(b, L.st[1], L.ss[1], b0, bs);
      for (int t = 2; t <= 4; ++t) pf_rows(b, L.st[t], L.ss[t], sl.lo, sl.n());
      return;
    }
    if (j == 1) {
      const Slice sl = slice_of(2 * mi, rank, CL);
      P1(b.take<WT>(size_t(sl.n()) * H), static_cast<const WT*>(L.w[9]) + size_t(sl.lo) * H, sl.n() * H * sizeof(WT));
      const int lo = min(sl.lo, mi), hi = min(sl.hi, mi), n = hi - lo;  // x_proj channels
      for (int t = 10; t <= 12; ++t) P1(b.take<float>(4 * n), static_cast<const float*>(L.w[t]) + 4 * lo, 4 * n * 4);
      P2(b.take<float>(4 * n), static_cast<const float*>(L.w[13]) + lo, 4, n * 4, mi * 4ll, n * 4);
      P1(b.take<float>(n), static_cast<const float*>(L.w[14]) + lo, n * 4);
      pf_conv(b, L.st[5], L.ss[5], mi, lo, hi);
      return;
    }
    if (j == 2) {
      const Slice sl = slice_of(mi, rank, CL);
      if (sl.n() == 0) return;  // no columns here: no head to read
      const int n = sl.lo / hs_x, k0 = sl.lo - n * hs_x;
      float* gw = b.take<float>(2 * 3 * mi);
      P1(gw, static_cast<const float*>(L.w[15]) + size_t(n) * 3 * mi, 3 * mi * 4);
      P1(gw + 3 * mi, static_cast<const float*>(L.w[15]) + size_t(nh_x + n) * 3 * mi, 3 * mi * 4);
      float* C = b.take<float>(RM * hs_x * sl.n());
      for (int r = 0; r < R; ++r)
        P2(C + size_t(r) * hs_x * sl.n(), L.st[6] + slot[r] * L.ss[6] + size_t(n) * hs_x * hs_x + k0, hs_x,
             sl.n() * 4, hs_x * 4ll, sl.n() * 4);
      pf_rows(b, L.st[7], L.ss[7], n * hs_x, hs_x);
      pf_rows(b, L.st[8], L.ss[8], n, 1);
      return;
    }
    const Slice sl = slice_of(H, rank, CL);
    P1(b.take<WT>(size_t(sl.n()) * mi), static_cast<const WT*>(L.w[19]) + size_t(sl.lo) * mi, sl.n() * mi * sizeof(WT));
  }

  __device__ void run_xlstm(int j, const LatLayer& L, Bump& b, const SV& sv) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (j == 0) {
      // sLSTM block (xlstm.py:297-320) for the CTA's channels, all in one sLSTM head block
      rmsnorm<WT>(a.X, a.ldH, H, R, sv.p[0], kF32Eps, a.U0, a.ldH, nullptr, 0, a.red);  // norm1 -> the layer input (skip)
      layernorm(a.U0, a.ldH, H, R, sv.p[1], 1e-5f, a.O1, a.ldH, a.red);  // O1 = LN(u) here (scratch until stage B)
      const Slice sl = slice_of(H, rank, CL);
      if (sl.n() == 0) return;  // the prologue above (U0, O1) is still this CTA's own
      const int jb = sl.lo / bs, b0 = jb * bs, n = sl.n();
      const float* wg = b.take<float>(size_t(n) * 2 * bs);  // gates i, f, z, o consecutive
      b.take<float>(size_t(n) * 2 * bs);
      b.take<float>(size_t(n) * 2 * bs);
      b.take<float>(size_t(n) * 2 * bs);
      const float* bias = b.take<float>(4 * n);
      const float* cw = b.take<float>(4 * bs);
      const float* cb = b.take<float>(bs);
      const float* cs = b.take<float>(RM * 3 * bs);
      const float* hp = b.take<float>(RM * bs);
      const float* cst = b.take<float>(RM * n);
      const float* nst = b.take<float>(RM * n);
      const float* mst = b.take<float>(RM * n);
      // gate inputs per row: xa = [silu(conv(LN u)) | h], xb = [LN u | h] over the head block
      float* xa = a.V2;                      // [R][2bs] (V2 is free until stage C)
      float* xb = a.V2 + RM * 2 * bs;
      for (int i = threadIdx.x; i < bs * R; i += kCThreads) {
        const int r = i / bs, k = i - r * bs, c = b0 + k;
        const float v = a.O1[r * a.ldH + c];
        const float* st = cs + r * 3 * bs;
        const float y = conv1(cw, bs, k, cb[k], st[k], st[bs + k], st[2 * bs + k], v);
        if (c >= sl.lo && c < sl.hi) {  // the channel's owner shifts its window
          float* g = L.st[0] + slot[r] * L.ss[0];
          g[c] = st[bs + k];
          g[H + c] = st[2 * bs + k];
          g[2 * H + c] = v;
        }
        xa[r * 2 * bs + k] = siluf_(y);
        xb[r * 2 * bs + k] = v;
        xa[r * 2 * bs + bs + k] = hp[r * bs + k];
        xb[r * 2 * bs + bs + k] = hp[r * bs + k];
      }
      csync();
      float* G = a.stg;  // [R][4n]
      gemv<float>(wg, 2 * bs, 2 * bs, 2 * n, xa, 2 * bs, R, G, 4 * n);             // i, f
      gemv<float>(wg + size_t(2) * n * 2 * bs, 2 * bs, 2 * bs, 2 * n, xb, 2 * bs, R, G + 2 * n, 4 * n);  // z, o
      csync();
      float* hout = a.stg + RM * 4 * n;
      for (int i = threadIdx.x; i < n * R; i += kCThreads) {
        const int r = i / n, e = i - r * n, c = sl.lo + e;
        const float* gr = G + r * 4 * n;
        float cc = cst[r * n + e], nn = nst[r * n + e], mm = mst[r * n + e];
        const float y = slstm_cell1(gr[e] + bias[e], gr[n + e] + bias[n + e], gr[2 * n + e] + bias[2 * n + e],
                                    gr[3 * n + e] + bias[3 * n + e], cc, nn, mm);
        L.st[1][slot[r] * L.ss[1] + c] = y;
        L.st[2][slot[r] * L.ss[2] + c] = cc;
        L.st[3][slot[r] * L.ss[3] + c] = nn;
        L.st[4][slot[r] * L.ss[4] + c] = mm;
        hout[r * n + e] = y;
      }
      csync();
      bcast(hout, n, n, R, a.HN, a.ldH, sl.lo, CL);
      return;
    }
    if (j == 1) {
      // O1 = GroupNorm(h) + u (xlstm.py:318-320); LN; x|gate projections; conv; q, k, v
      group_stats(a.HN, a.ldH, nbl, bs, R, 1e-5f, a.gm, a.gr);
      const float* gnw = sv.p[1];
      const float* gnb = sv.p[2];
      for (int i = threadIdx.x; i < H * R; i += kCThreads) {
        const int r = i / H, e = i - r * H, g = e / bs;
        const float y = (a.HN[r * a.ldH + e] - a.gm[r * nbl + g]) * a.gr[r * nbl + g];
        a.O1[r * a.ldH + e] = (y * gnw[e] + gnb[e]) + a.U0[r * a.ldH + e];
      }
      csync();
      float* T = a.T;
      const int ldT = a.ldT;
      layernorm_to(a.O1, a.ldH, H, R, sv.p[3], 1e-5f, [=](int r, int e, float y) { T[r * ldT + e] = WVec<WT>::round(y); }, a.red);
      const Slice sl = slice_of(2 * mi, rank, CL);
      const WT* w = b.take<WT>(size_t(sl.n()) * H);
      const int lo = min(sl.lo, mi), hi = min(sl.hi, mi), n = hi - lo;
      const float* wq = b.take<float>(4 * n);
      const float* wk = b.take<float>(4 * n);
      const float* wv = b.take<float>(4 * n);
      const float* cw = b.take<float>(4 * n);
      const float* cb = b.take<float>(n);
      const float* cs = b.take<float>(RM * 3 * n);
      const int ld = rup4(sl.n());
      gemv<WT>(w, H, H, sl.n(), a.T, a.ldT, R, a.stg, ld);
      csync();
      // x rows: xm (rounded), xc = silu(conv(xm)); gate rows: xg (rounded)
      float* xcv = a.stg + RM * ld;  // [R][n] conv+SiLU of the x rows
      for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
        const int r = i / sl.n(), e = i - r * sl.n(), idx = sl.lo + e;
        float v = WVec<WT>::round(a.stg[r * ld + e]);
        a.stg[r * ld + e] = v;
        if (idx < mi) {
          const int k = idx - lo;
          const float* st = cs + r * 3 * n;
          const float y = conv1(cw, n, k, cb[k], st[k], st[n + k], st[2 * n + k], v);
          float* g = L.st[5] + slot[r] * L.ss[5];
          g[idx] = st[n + k];
          g[mi + idx] = st[2 * n + k];
          g[2 * mi + idx] = v;
          xcv[r * n + k] = siluf_(y);
        }
      }
      csync();
      // q, k from xc and v from xm: 4x4 blocks (BlockLinear, model/modules.py:71-79)
      float* qkv = xcv + RM * rup4(n);  // [R][3][n]
      for (int i = threadIdx.x; i < n * R; i += kCThreads) {
        const int r = i / n, k = i - r * n, q4 = k & ~3, o = k & 3;
        const float* xc = xcv + r * n + q4;
        const float* xm = a.stg + r * ld + (lo - sl.lo) + q4;
        float qv = 0.f, kv = 0.f, vv = 0.f;
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          qv = fmaf(wq[(q4 + o) * 4 + h], xc[h], qv);
          kv = fmaf(wk[(q4 + o) * 4 + h], xc[h], kv);
          vv = fmaf(wv[(q4 + o) * 4 + h], xm[h], vv);
        }
        qkv[(r * 3 + 0) * n + k] = qv;
        qkv[(r * 3 + 1) * n + k] = kv;
        qkv[(r * 3 + 2) * n + k] = vv;
      }
      csync();
      if (n > 0) {
        bcast(xcv, n, n, R, a.V1, a.ld1, lo, CL);  // xc
        for (int t = 0; t < 3; ++t)  // q, k, v: row r of each at qkv + (3r + t) n
          bcast(qkv + t * n, 3 * n, n, R, a.V1, a.ld1, (2 + t) * mi + lo, CL);
      }
      const int glo = max(sl.lo, mi), ghi = max(sl.hi, mi);
      if (ghi > glo) {  // gate rows -> xg at [mi, 2mi)
        cg::cluster_group cluster = cg::this_cluster();
        for (int i = threadIdx.x; i < CL * R * (ghi - glo); i += kCThreads) {
          const int peer = i / (R * (ghi - glo)), rem = i - peer * R * (ghi - glo), r = rem / (ghi - glo),
                    k = rem - r * (ghi - glo);
          *cluster.map_shared_rank(a.V1 + r * a.ld1 + glo + k, peer) = a.stg[r * ld + (glo - sl.lo) + k];
        }
      }
      return;
    }
    if (j == 2) {
      // mLSTM cell for the CTA's columns of one head (xlstm.py:55-133)
      const Slice sl = slice_of(mi, rank, CL);
      if (sl.n() == 0) return;  // no columns of any head here
      const int n = sl.lo / hs_x, k0 = sl.lo - n * hs_x, nc = sl.n();
      const float* gw = b.take<float>(2 * 3 * mi);
      const float* C = b.take<float>(RM * hs_x * nc);
      const float* nold = b.take<float>(RM * hs_x);
      const float* mold = b.take<float>(RM);
      const float* gb = sv.p[1];
      float* pre = a.gm;  // [R][2]: i, f pre-activations
      dot2_wide(gw, 3 * mi, 3 * mi, a.V1 + 2 * mi, a.ld1, R, pre, a.red);  // igate|fgate over [q;k;v] (fp32)
      // stabiliser and gates (xlstm.py:88-96); n (xlstm.py:101-105); q.n
      float* ks = a.stg;                          // [R][hs] k / sqrt(hs)
      float* nn = a.stg + RM * hs_x;     // [R][hs] new n
      float* gf = a.stg + 2 * RM * hs_x; // [R][4]: i, f, m_new, den
      if (threadIdx.x < R) {
        const int r = threadIdx.x;
        const float ig = pre[r * 2] + gb[n], fg = pre[r * 2 + 1] + gb[nh_x + n];
        const float mo = mold[r];
        const float lf = logsigmoidf_(fg);
        const float mn = fmaxf(ig, mo + lf);
        gf[r * 4 + 0] = expf(ig - mn);
        gf[r * 4 + 1] = expf(lf + mo - mn);
        gf[r * 4 + 2] = mn;
      }
      csync();
      const float sq = sqrtf(float(hs_x));
      for (int i = threadIdx.x; i < hs_x * R; i += kCThreads) {
        const int r = i / hs_x, h = i - r * hs_x;
        const float k = a.V1[r * a.ld1 + 3 * mi + n * hs_x + h] / sq;  // k / sqrt(head_size) (xlstm.py:99)
        ks[r * hs_x + h] = k;
        nn[r * hs_x + h] = gf[r * 4 + 1] * nold[r * hs_x + h] + gf[r * 4 + 0] * k;
      }
      csync();
      for (int r = warp; r < R; r += kCWarps) {
        float qn = 0.f;
        for (int h = lane; h < hs_x; h += 32) qn = fmaf(a.V1[r * a.ld1 + 2 * mi + n * hs_x + h], nn[r * hs_x + h], qn);
        qn = warp_sum(qn);
        if (lane == 0) gf[r * 4 + 3] = fmaxf(fabsf(qn), expf(-gf[r * 4 + 2])) + 1e-6f;  // xlstm.py:130-132
      }
      if (k0 == 0) {  // the head's first CTA writes n and m
        for (int i = threadIdx.x; i < hs_x * R; i += kCThreads) {
          const int r = i / hs_x, h = i - r * hs_x;
          L.st[7][slot[r] * L.ss[7] + n * hs_x + h] = nn[r * hs_x + h];
        }
        if (threadIdx.x < R) L.st[8][slot[threadIdx.x] * L.ss[8] + n] = gf[threadIdx.x * 4 + 2];
      }
      csync();
      // C = f*C + (i*k) v; num = q.C per column (xlstm.py:108-118)
      float* out = a.stg + 2 * RM * hs_x + 4 * RM;
      for (int pc = warp; pc < nc * R; pc += kCWarps) {
        const int r = pc / nc, c = pc - r * nc, col = k0 + c;
        const float ig = gf[r * 4 + 0], fg = gf[r * 4 + 1];
        const float v = a.V1[r * a.ld1 + 4 * mi + n * hs_x + col];
        float* g = L.st[6] + slot[r] * L.ss[6] + size_t(n) * hs_x * hs_x + col;
        float num = 0.f;
        for (int h = lane; h < hs_x; h += 32) {
          const float cn = fg * C[(size_t(r) * hs_x + h) * nc + c] + (ig * ks[r * hs_x + h]) * v;
          g[size_t(h) * hs_x] = cn;
          num = fmaf(a.V1[r * a.ld1 + 2 * mi + n * hs_x + h], cn, num);
        }
        num = warp_sum(num);
        if (lane == 0) out[r * nc + c] = num / gf[r * 4 + 3];  // xlstm.py:133
      }
      csync();
      bcast(out, nc, nc, R, a.V2, a.ld2, sl.lo, CL);
      return;
    }
    // D: GroupNorm per head; + skip * xc; * silu(xg); proj_down + O1 (xlstm.py:143-147, 216-220)
    group_stats(a.V2, a.ld2, nh_x, hs_x, R, 1e-5f, a.gm, a.gr);
    const float* ow = sv.p[1];
    const float* ob = sv.p[2];
    const float* skip = sv.p[3];
    for (int i = threadIdx.x; i < mi * R; i += kCThreads) {
      const int r = i / mi, e = i - r * mi, g = e / hs_x;
      const float y = (a.V2[r * a.ld2 + e] - a.gm[r * nh_x + g]) * a.gr[r * nh_x + g] * ow[e] + ob[e];
      const float* v1 = a.V1 + r * a.ld1;
      a.T[r * a.ldT + e] = WVec<WT>::round((y + skip[e] * v1[e]) * siluf_(v1[mi + e]));
    }
    csync();
    const Slice sl = slice_of(H, rank, CL);
    const WT* w = b.take<WT>(size_t(sl.n()) * mi);
    const int ld = rup4(sl.n());
    gemv<WT>(w, mi, mi, sl.n(), a.T, a.ldT, R, a.stg, ld);
    csync();
    for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
      const int r = i / sl.n(), e = i - r * sl.n();
      a.stg[r * ld + e] = WVec<WT>::round(a.stg[r * ld + e]) + a.O1[r * a.ldH + sl.lo + e];
    }
    csync();
    bcast(a.stg, ld, sl.n(), R, a.OUT2, a.ldH, sl.lo, CL);
  }

  // =============================================================== run

  __device__ void run(int s, uint8_t* buf) {
    Bump b{buf};
    if (s == 0) {
      // input_up: relu(CastLinear(features)) (model/inference_model.py:88)
      for (int i = threadIdx.x; i < R * fpad; i += kCThreads) {
        const int r = i / fpad, k = i - r * fpad;
        a.T[r * a.ldT + k] = k < F ? WVec<WT>::round(io.feats[r * F + k]) : 0.f;
      }
      csync();
      const Slice sl = slice_of(P, rank, CL);
      const WT* w = b.take<WT>(sl.n() * fpadw());
      const WT* bias = b.take<WT>(sl.n());
      const int ld = rup4(sl.n());
      gemv<WT>(w, fpadw(), fpad, sl.n(), a.T, a.ldT, R, a.stg, ld);
      csync();
      for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
        const int r = i / sl.n(), e = i - r * sl.n();
        a.stg[r * ld + e] = fmaxf(WVec<WT>::round(a.stg[r * ld + e] + WVec<WT>::one(bias, e)), 0.f);
      }
      csync();
      bcast(a.stg, ld, sl.n(), R, a.U1, a.ldP, sl.lo, CL);
      return;
    }
    if (s == 1) {
      // input_down (model/inference_model.py:89)
      const Slice sl = slice_of(H, rank, CL);
      const WT* w = b.take<WT>(size_t(sl.n()) * P);
      const WT* bias = b.take<WT>(sl.n());
      const int ld = rup4(sl.n());
      gemv<WT>(w, P, P, sl.n(), a.U1, a.ldP, R, a.stg, ld);
      csync();
      for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
        const int r = i / sl.n(), e = i - r * sl.n();
        a.stg[r * ld + e] = WVec<WT>::round(a.stg[r * ld + e] + WVec<WT>::one(bias, e));
      }
      csync();
      bcast(a.stg, ld, sl.n(), R, a.X, a.ldH, sl.lo, CL);
      return;
    }
    const int blk = (s - 2) / per_block(), j = (s - 2) % per_block();
    const LatBlock& B = blocks[blk];
    const SV v = small_vecs(j, B, b, false);
    if (j == per_block() - 2) {
      // MLP1: (xLSTM: X += LayerNorm(OUT2), xlstm.py:365) fc1 + ReLU on norm2(X) (inference_model.py:64-65)
      const float* xin = a.X;
      if (kind == kXLSTM) {
        float* Xa = a.Xa;
        const float* X = a.X;
        const int ld = a.ldH;
        // y + x (inference_model.py:64), rounded as a separate add after the norm
        layernorm_to(a.OUT2, ld, H, R, v.p[1], 1e-5f, [=](int r, int e, float y) { Xa[r * ld + e] = __fadd_rn(y, X[r * ld + e]); }, a.red);
        xin = a.Xa;
      }
      rmsnorm<WT>(xin, a.ldH, H, R, v.p[0], kF32Eps, nullptr, 0, a.T, a.ldT, a.red);
      const Slice sl = slice_of(P, rank, CL);
      const WT* w = b.take<WT>(size_t(sl.n()) * H);
      const WT* bias = b.take<WT>(sl.n());
      const int ld = rup4(sl.n());
      gemv<WT>(w, H, H, sl.n(), a.T, a.ldT, R, a.stg, ld);
      csync();
      for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
        const int r = i / sl.n(), e = i - r * sl.n();
        a.stg[r * ld + e] = fmaxf(WVec<WT>::round(a.stg[r * ld + e] + WVec<WT>::one(bias, e)), 0.f);
      }
      csync();
      bcast(a.stg, ld, sl.n(), R, a.Y, a.ldP, sl.lo, CL);
      return;
    }
    if (j == per_block() - 1) {
      // MLP2: X + fc2(Y) (inference_model.py:65)
      const Slice sl = slice_of(H, rank, CL);
      const WT* w = b.take<WT>(size_t(sl.n()) * P);
      const WT* bias = b.take<WT>(sl.n());
      const float* xres = kind == kXLSTM ? a.Xa : a.X;
      const int ld = rup4(sl.n());
      gemv<WT>(w, P, P, sl.n(), a.Y, a.ldP, R, a.stg, ld);
      csync();
      for (int i = threadIdx.x; i < sl.n() * R; i += kCThreads) {
        const int r = i / sl.n(), e = i - r * sl.n();
        a.stg[r * ld + e] = xres[r * a.ldH + sl.lo + e] + WVec<WT>::round(a.stg[r * ld + e] + WVec<WT>::one(bias, e));
      }
      csync();
      bcast(a.stg, ld, sl.n(), R, a.X, a.ldH, sl.lo, CL);
      return;
    }
    switch (kind) {
      case kMamba2: return run_mamba(j, B.L, b, v);
      case kRetNet: return run_retnet(j, B.L, b, v);
      case kHawk: return run_hawk(j, B.L, b, v);
      default: return run_xlstm(j, B.L, b, v);
    }
  }
};

// One tower's whole step on its cluster: the producer warp copies stage s+1's
// slice (16- and 4-byte cp.async) while the compute warps run stage s, the
// stages separated by cluster barriers, then output_proj of the tower's column.
template <class WT, int KIND, int RT>
__device__ __noinline__ void tower_main(const LatModel& M, const LatIO& io, uint8_t* smem, int rank, int CL) {
  Tower<WT, KIND, RT> tw(M, M.t[KIND], io, rank, CL, smem);
  tw.load_desc();
  const uint32_t act_bytes = M.act_bytes[KIND], buf_bytes = M.buf_bytes[KIND];  // this tower's carve
  uint8_t* buf[2] = {smem + act_bytes, smem + act_bytes + buf_bytes};
  const int ns = tw.nstages();
  if (KIND == 0 && rank == 0 && threadIdx.x == 0 && io.err_out) *io.err_out = *M.err;
  // the producer warp loads output_proj's weights and the first stage's slice
  if (rank == 0) pf1d(tw.a.OW, M.ow, tw.H * 4);
  tw.prefetch(0, buf[0]);
  cp_commit();
  cp_wait_all();
  __syncthreads();
  cluster_arrive();
#ifdef B2E_LAT_TRACE
  // cluster rank 0's thread 0 (compute) and first producer lane stamp each stage
  const bool trc = rank == 0 && threadIdx.x == 0, trp = rank == 0 && threadIdx.x == kCThreads;
  unsigned long long ts[kTraceFields] = {};
#define B2E_STAMP(i) \
  if (trc || trp) ts[i] = gtime()
#else
#define B2E_STAMP(i)
#endif
  const bool producer = threadIdx.x >= kCThreads;
  for (int s = 0; s < ns; ++s) {
    B2E_STAMP(0);
    cluster_wait();  // every CTA's outputs of stage s-1 are in this CTA's shared memory
    B2E_STAMP(1);
    uint32_t nb = 0;
    if (producer) {
      // the next stage's slice, beside this stage's work (its buffer was last
      // read by stage s-1, finished before the barrier that ended it)
      if (s + 1 < ns) nb = tw.prefetch(s + 1, buf[(s + 1) & 1]);
      cp_commit();
      cp_wait_all();
    } else {
      tw.run(s, buf[s & 1]);
    }
    (void)nb;
    B2E_STAMP(2);  // compute: the stage's work done; producer: the copies landed
    B2E_STAMP(3);
    // Every thread of every CTA arrives (release) and, at the next stage's start,
    // waits (acquire): this CTA's stage-s work and the producer's copies of stage
    // s+1 are visible to all its threads then, and stage s's buffer is free for
    // the copies of stage s+2. No CTA barrier is needed besides.
    cluster_arrive();
    B2E_STAMP(4);
#ifdef B2E_LAT_TRACE
    if (s < kTraceStages) {
      unsigned long long* g = g_lat_trace[KIND][s];
      if (trc) {
        g[0] = ts[0]; g[1] = ts[1]; g[2] = ts[2]; g[4] = ts[3]; g[5] = ts[4];
      }
      if (trp) {
        g[3] = ts[2];
        g[6] = nb;  // bytes of stage s+1's copies
      }
    }
#endif
  }
#undef B2E_STAMP
  cluster_wait();
  cp_wait_all();
  // output_proj of this tower's column (model/inference_model.py:142), f32
  if (rank == 0) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int r = warp; r < tw.R; r += kWarps) {
      float acc = 0.f;
      for (int k = lane; k < tw.H; k += 32) acc = fmaf(tw.a.OW[k], tw.a.X[r * tw.a.ldH + k], acc);
      acc = warp_sum(acc);
      if (lane == 0) io.preds[r * 4 + KIND] = acc + M.ob[0];
    }
  }
}

template <class WT, int RT>
__global__ void __launch_bounds__(kThreads, 1) k_latency_step(const LatModel* __restrict__ model,
                                                               const __grid_constant__ LatIO io) {
  extern __shared__ __align__(16) uint8_t smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int CL = int(cluster.num_blocks());
  const int rank = int(cluster.block_rank());
  switch (blockIdx.x / CL) {  // cluster t runs tower t (xLSTM, Mamba2, RetNet, Hawk)
    case 0: tower_main<WT, kXLSTM, RT>(*model, io, smem, rank, CL); break;
    case 1: tower_main<WT, kMamba2, RT>(*model, io, smem, rank, CL); break;
    case 2: tower_main<WT, kRetNet, RT>(*model, io, smem, rank, CL); break;
    default: tower_main<WT, kHawk, RT>(*model, io, smem, rank, CL); break;
  }
}

// Planning pass: the shared memory the kernel carves (activations; the largest
// stage buffer over every stage, rank and tower) for the worst-case row count,
// measured by running the kernel's own carving code with no copies issued.
template <class WT, int KIND>
__device__ void plan_tower(const LatModel& M, int CL, uint32_t* out) {
  LatIO io{};
  io.n = M.rmax;
  uint32_t act = 0, buf = 0;
  for (int rank = 0; rank < CL; ++rank) {
    Tower<WT, KIND, 0> tw(M, M.t[KIND], io, rank, CL, nullptr);
    long long zero_slots[kLatMaxRows] = {};
    tw.slot = zero_slots;  // addresses are formed, nothing is read through them
    tw.dry = true;
    act = max(act, tw.act_used);
    for (int s = 0; s < tw.nstages(); ++s) buf = max(buf, tw.prefetch(s, nullptr));
  }
  out[2 * KIND] = act;
  out[2 * KIND + 1] = (buf + 127u) & ~127u;
}

template <class WT>
__global__ void k_latency_plan(const LatModel* __restrict__ model, int CL, uint32_t* out) {
  plan_tower<WT, kXLSTM>(*model, CL, out);
  plan_tower<WT, kMamba2>(*model, CL, out);
  plan_tower<WT, kRetNet>(*model, CL, out);
  plan_tower<WT, kHawk>(*model, CL, out);
}

}  // namespace

// ----------------------------------------------------------------- host

namespace {

template <class WT>
void* kernel_of(int rt) {
  return rt ? reinterpret_cast<void*>(k_latency_step<WT, 1>) : reinterpret_cast<void*>(k_latency_step<WT, 0>);
}

void* step_kernel(int lp, int rt) {
  return lp == kBF16 ? kernel_of<__nv_bfloat16>(rt) : lp == kF16 ? kernel_of<__half>(rt) : kernel_of<float>(rt);
}

}  // namespace

LatencyPath::LatencyPath(const Dims& d, int lp, const LatTower (&towers)[4],
                         const std::vector<std::vector<LatBlock>>& blocks, const float* ow, const float* ob, int* err)
    : lp_(lp) {
  if (d.F > kLatMaxFeatures) {
    why_ = "more than " + std::to_string(kLatMaxFeatures) + " features";
    return;
  }
  if (d.P % 4 != 0 || d.H % 4 != 0) {
    why_ = "hidden and proj sizes must be multiples of 4";
    return;
  }
  if (d.heads < 4) {  // the sLSTM gate inputs of a stage share the mLSTM output buffer
    why_ = "fewer than 4 heads";
    return;
  }
  // device descriptors
  LatModel m{};
  m.rmax = kLatMaxRows;
  m.H = d.H; m.P = d.P; m.F = d.F; m.fpad = lp == kF32 ? d.F : (d.F + 7) & ~7; m.depth = d.depth; m.lp = lp;
  m.heads = d.heads; m.m_hs = d.m_hs; m.m_bc = d.m_bc;
  m.ow = ow; m.ob = ob; m.err = err;
  std::vector<LatBlock> all;
  for (int t = 0; t < 4; ++t) all.insert(all.end(), blocks[t].begin(), blocks[t].end());
  B2E_CUDA(cudaMalloc(&d_blocks_, all.size() * sizeof(LatBlock)));
  B2E_CUDA(cudaMemcpy(d_blocks_, all.data(), all.size() * sizeof(LatBlock), cudaMemcpyHostToDevice));
  for (int t = 0; t < 4; ++t) {
    m.t[t] = towers[t];
    m.t[t].blocks = d_blocks_ + size_t(t) * d.depth;
  }
  B2E_CUDA(cudaMalloc(&d_model_, sizeof(LatModel)));
  B2E_CUDA(cudaMemcpy(d_model_, &m, sizeof(LatModel), cudaMemcpyHostToDevice));
  uint32_t* d_plan = nullptr;
  B2E_CUDA(cudaMalloc(&d_plan, 32));
  int dev = 0, max_smem = 0;
  B2E_CUDA(cudaGetDevice(&dev));
  B2E_CUDA(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
  for (int CL : {16, 8})
    for (int rmax : {kLatMaxRows, 2, 1}) {
    if (ok_) break;
    // the stage plan keeps a CTA's columns inside one sLSTM head block and one mLSTM head
    auto chunk = [&](int N) { return ((N + CL - 1) / CL + 3) & ~3; };
    const int bs = d.H / (d.heads / 2), hsx = 2 * d.H / d.heads;
    if (chunk(d.H) > bs || bs % chunk(d.H) != 0) {
      why_ = "sLSTM head blocks do not hold whole slices";
      continue;
    }
    if (chunk(2 * d.H) > hsx || hsx % chunk(2 * d.H) != 0) {
      why_ = "mLSTM heads do not hold whole slices";
      continue;
    }
    m.rmax = rmax;
    B2E_CUDA(cudaMemcpy(d_model_, &m, sizeof(LatModel), cudaMemcpyHostToDevice));
    uint32_t plan[8] = {};
    if (lp == kBF16)
      k_latency_plan<__nv_bfloat16><<<1, 1>>>(d_model_, CL, d_plan);
    else if (lp == kF16)
      k_latency_plan<__half><<<1, 1>>>(d_model_, CL, d_plan);
    else
      k_latency_plan<float><<<1, 1>>>(d_model_, CL, d_plan);
    B2E_CUDA(cudaGetLastError());
    B2E_CUDA(cudaMemcpy(plan, d_plan, 32, cudaMemcpyDeviceToHost));
    size_t smem = 0;  // the launch gives every CTA the largest tower's carve
    for (int t = 0; t < 4; ++t) {
      m.act_bytes[t] = plan[2 * t];
      m.buf_bytes[t] = plan[2 * t + 1];
      smem = std::max(smem, size_t(plan[2 * t]) + 2 * size_t(plan[2 * t + 1]));
    }
    if (smem > size_t(max_smem)) {
      why_ = "stage slices need " + std::to_string(smem) + " bytes of shared memory";
      continue;
    }
    void* kern = step_kernel(lp, 0);
    bool refused = false;
    for (int rt = 0; rt < 2; ++rt) {
      void* k = step_kernel(lp, rt);
      if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess ||
          (CL > 8 && cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess))
        refused = true;
    }
    if (refused) {
      cudaGetLastError();
      why_ = "cluster of " + std::to_string(CL) + " refused";
      continue;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(4 * CL);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = CL;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1) {
      cudaGetLastError();
      why_ = "cluster of " + std::to_string(CL) + " cannot be scheduled";
      continue;
    }
    B2E_CUDA(cudaMemcpy(d_model_, &m, sizeof(LatModel), cudaMemcpyHostToDevice));  // with the carve sizes
    cl_ = CL;
    smem_ = smem;
    rows_ = rmax;
    clusters_ = clusters;
    ok_ = true;
    break;
  }
  cudaFree(d_plan);
}

LatencyPath::~LatencyPath() {
  if (d_model_) cudaFree(d_model_);
  if (d_blocks_) cudaFree(d_blocks_);
}

void LatencyPath::launch(const LatIO& io, cudaStream_t s) const {
  B2E_CHECK(ok_, kErrInternal, "latency path unavailable: " + why_);
  B2E_CHECK(io.n >= 1 && io.n <= rows_, kErrInvalid, "latency step of " + std::to_string(io.n) + " rows");
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(4 * cl_);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem_;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cl_;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const LatModel* m = d_model_;
  const bool one = io.n == 1;  // the single-request kernel: every row loop folded to one row
  if (lp_ == kBF16)
    B2E_CUDA(one ? cudaLaunchKernelEx(&cfg, k_latency_step<__nv_bfloat16, 1>, m, io)
                 : cudaLaunchKernelEx(&cfg, k_latency_step<__nv_bfloat16, 0>, m, io));
  else if (lp_ == kF16)
    B2E_CUDA(one ? cudaLaunchKernelEx(&cfg, k_latency_step<__half, 1>, m, io)
                 : cudaLaunchKernelEx(&cfg, k_latency_step<__half, 0>, m, io));
  else
    B2E_CUDA(one ? cudaLaunchKernelEx(&cfg, k_latency_step<float, 1>, m, io)
                 : cudaLaunchKernelEx(&cfg, k_latency_step<float, 0>, m, io));
}

}  // namespace b2e

#ifdef B2E_LAT_TRACE
// Profiling build only: the last step's stage stamps, [4 towers][512 stages][8]
// u64 (stage start, cluster barrier passed, compute warps' work done, producer's
// copies of the next stage landed, CTA barrier passed, arrived, next stage's
// bytes, 0); returns a cudaError_t.
extern "C" __attribute__((visibility("default"))) int b2e_lat_trace_read(void* host) {
  return int(cudaMemcpyFromSymbol(host, b2e::g_lat_trace, sizeof(b2e::g_lat_trace)));
}
#endif
