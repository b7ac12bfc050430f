// The four recurrent layers (xLSTM, Mamba2, RetNet, Hawk) on sm_100a.
//
// Each layer step is a short chain: projection GEMM(s) -> one per-row fused
// kernel (convs, gates, norms, rotary) -> the state-streaming cell kernel over
// the big state (cells.cu) -> one per-row fused kernel -> output GEMM with the
// Block residual in its epilogue. Every per-row kernel is one CTA per live row,
// reads and writes the row's small state leaves in place at its slot, and keeps
// the row's intermediate vectors in shared memory. The arithmetic of every step
// is the reference's, in its order, in float32; the citations give the lines.
#include <algorithm>
#include <cmath>

#include "cells.cuh"
#include "gemm.cuh"
#include "layers.cuh"
#include "latency.cuh"

namespace b2e {


void Dims::validate() const {
  B2E_CHECK(H > 0 && P > 0 && depth > 0 && F > 0, kErrInvalid, "model dims must be positive");
  B2E_CHECK(heads >= 2 && heads % 2 == 0, kErrInvalid, "num_heads must be even (sLSTM uses num_heads // 2)");
  B2E_CHECK(heads <= 64, kErrInvalid, "num_heads above 64 is not supported (per-row group statistics)");
  B2E_CHECK(H % heads == 0 && H % (heads / 2) == 0 && H % 4 == 0, kErrInvalid, "hidden_size must divide by heads and 4");
  B2E_CHECK((2 * H) % m_hs == 0, kErrInvalid, "mamba inner size must divide by its head size");
  B2E_CHECK(retnet_hs() % 2 == 0, kErrInvalid, "RetNet head size must be even (rotary pairs)");
  B2E_CHECK(retnet_hs() % 4 == 0 && mlstm_hs() % 4 == 0 && m_bc % 4 == 0, kErrInvalid,
            "head sizes and the Mamba2 B/C width must be multiples of 4");
  B2E_CHECK(retnet_hs() <= 512 && mlstm_hs() <= 512, kErrInvalid, "head sizes above 512 are not supported");
}

const char* layer_name(int kind) {
  switch (kind) {
    case kXLSTM: return "xlstm";
    case kMamba2: return "mamba2";
    case kRetNet: return "retnet";
    case kHawk: return "hawk";
  }
  return "?";
}

namespace {

constexpr int kRowThreads = 256;
// Per-row kernels walk a row in chunks of kEU elements per thread and issue all
// of a chunk's loads before its first store: a load placed after a store waits
// for it (the compiler cannot tell the stores from the loads' sources), which
// at hidden 2048 made a row loop a chain of one memory round trip per element.
constexpr int kEU = 8;

struct RowCtx {
  const int* n_dev;
  int rows;
  const int* slots;
};

__device__ __forceinline__ bool row_live(const RowCtx& r, int row) { return row < live_rows(r.n_dev, r.rows); }
__device__ __forceinline__ long long row_slot(const RowCtx& r, int row) { return r.slots ? r.slots[row] : row; }

// nn.Conv1d(C, C, 4, groups=C) on the window [state (3 taps), x] (model/modules.py:37-41).
// Weights are stored tap-major (4, C); the state row is (3, C).
__device__ __forceinline__ float conv_step(const float* w, const float* bias, float* st, int C, int c, float x) {
  const float s0 = st[c], s1 = st[C + c], s2 = st[2 * C + c];
  float acc = w[c] * s0;
  acc = fmaf(w[C + c], s1, acc);
  acc = fmaf(w[2 * C + c], s2, acc);
  acc = fmaf(w[3 * C + c], x, acc);
  st[c] = s1;
  st[C + c] = s2;
  st[2 * C + c] = x;
  return acc + bias[c];
}

// Mean and 1/sqrt(var + eps) of G groups of gs consecutive values; one warp per
// group, deterministic order. Results in smem gm[g], gr[g]; ends with a barrier.
__device__ void group_stats(const float* v, int G, int gs, float eps, float* gm, float* gr) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int g = w; g < G; g += nw) {
    const float* x = v + size_t(g) * gs;
    float s = 0.f;
    for (int i = lane; i < gs; i += 32) s += x[i];
    const float mu = warp_sum(s) / float(gs);
    float q = 0.f;
    for (int i = lane; i < gs; i += 32) {
      const float d = x[i] - mu;
      q = fmaf(d, d, q);
    }
    q = warp_sum(q) / float(gs);
    if (lane == 0) {
      gm[g] = mu;
      gr[g] = 1.0f / sqrtf(q + eps);
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------ Block glue

struct RmsP {
  RowCtx rc;
  const float* x; const float* w; float* out; int H; float eps; void* out_lp; int lp;
};
// One warp per row: H is a multiple of 4 (Dims::validate), so each lane moves
// 16-byte vectors; 8 rows per 256-thread CTA.
constexpr int kRowsPerCta = 8;

__global__ void __launch_bounds__(256) k_rmsnorm(const RmsP p) {
  prefetch_l1(p.w, p.H);
  pdl_wait();
  const int r = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (!row_live(p.rc, r)) return;
  const float4* x = reinterpret_cast<const float4*>(p.x + size_t(r) * p.H);
  const int n4 = p.H >> 2;
  constexpr int V = 16;  // rows of up to 32*V vectors (hidden 2048) stay in registers
  if (n4 <= 32 * V) {
    // every load of the row and of the weights in flight at once, before any
    // store (a load after a store waits for it: the compiler cannot tell that
    // the output does not alias the weights)
    float4 v[V], wv[V];
    float ss = 0.f;
    const float4* w4 = reinterpret_cast<const float4*>(p.w);
#pragma unroll
    for (int t = 0; t < V; ++t) {
      const int i = lane + 32 * t;
      v[t] = i < n4 ? x[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      wv[t] = (i < n4 && w4) ? w4[i] : make_float4(1.f, 1.f, 1.f, 1.f);
    }
#pragma unroll
    for (int t = 0; t < V; ++t) ss = fmaf(v[t].x, v[t].x, fmaf(v[t].y, v[t].y, fmaf(v[t].z, v[t].z, fmaf(v[t].w, v[t].w, ss))));
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(p.H) + p.eps);
#pragma unroll
    for (int t = 0; t < V; ++t) {
      const int i = lane + 32 * t;
      if (i >= n4) break;
      const float4 w = wv[t];
      const float4 o = make_float4(v[t].x * inv * w.x, v[t].y * inv * w.y, v[t].z * inv * w.z, v[t].w * inv * w.w);
      if (p.out) reinterpret_cast<float4*>(p.out + size_t(r) * p.H)[i] = o;
      if (p.out_lp) {
        const size_t base = size_t(r) * p.H + size_t(i) * 4;
        store_as(p.lp, p.out_lp, base + 0, o.x);
        store_as(p.lp, p.out_lp, base + 1, o.y);
        store_as(p.lp, p.out_lp, base + 2, o.z);
        store_as(p.lp, p.out_lp, base + 3, o.w);
      }
    }
    return;
  }
  float ss = 0.f;
  for (int i = lane; i < n4; i += 32) {
    const float4 v = x[i];
    ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / float(p.H) + p.eps);
  for (int i = lane; i < n4; i += 32) {
    const float4 v = x[i];
    const float4 w = p.w ? reinterpret_cast<const float4*>(p.w)[i] : make_float4(1.f, 1.f, 1.f, 1.f);
    const float4 o = make_float4(v.x * inv * w.x, v.y * inv * w.y, v.z * inv * w.z, v.w * inv * w.w);
    if (p.out) reinterpret_cast<float4*>(p.out + size_t(r) * p.H)[i] = o;
    if (p.out_lp) {
      const size_t base = size_t(r) * p.H + size_t(i) * 4;
      store_as(p.lp, p.out_lp, base + 0, o.x);
      store_as(p.lp, p.out_lp, base + 1, o.y);
      store_as(p.lp, p.out_lp, base + 2, o.z);
      store_as(p.lp, p.out_lp, base + 3, o.w);
    }
  }
}

struct OutP {
  RowCtx rc;
  const float* x; const float* w; const float* b; int H; float* preds; int ld; int col;
};
__global__ void __launch_bounds__(256) k_output_proj(const OutP p) {
  pdl_wait();
  const int r = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (!row_live(p.rc, r)) return;
  const float4* x = reinterpret_cast<const float4*>(p.x + size_t(r) * p.H);
  const float4* w = reinterpret_cast<const float4*>(p.w);
  float s = 0.f;
  for (int i = lane; i < (p.H >> 2); i += 32) {
    const float4 a = x[i], b = w[i];
    s = fmaf(a.x, b.x, fmaf(a.y, b.y, fmaf(a.z, b.z, fmaf(a.w, b.w, s))));
  }
  s = warp_sum(s);
  if (lane == 0) p.preds[size_t(r) * p.ld + p.col] = s + p.b[0];
}

__global__ void k_set_rows(int* n, int v) { *n = v; }

// ---------------------------------------------------------------- Mamba2
// model/mamba2.py:62-168.

struct Mamba2PreP {
  RowCtx rc;
  const float* proj; int ldp; int mi, bc, nh;  // proj row: [x (mi) | z (mi) | b (bc) | c (bc)]
  const float* tin; int H;                     // the layer input (norm1 output, f32) [row][H]
  const float* dtw; const float* dtb;          // dt_proj (fp32 kept): [nh][H], [nh]
  float* xconv; long long xcs; float* bconv; long long bcs; float* cconv; long long ccs;
  const float *wx, *bx, *wb, *bb, *wc, *bcv, *a;
  float *xs, *bs, *cs, *dt, *dc;
};
// Mamba2 between in_proj and the state step, kM2Rows rows per CTA: the three
// convs + SiLU and dt_proj with softplus and the decay. Every row's conv taps
// and inputs are loaded before any is updated (one round trip to memory per
// phase), conv and dt weights are shared by the CTA's rows.
constexpr int kM2Rows = 4;
// Conv + SiLU of channel i (< mi + 2bc: x, then b, then c) for rows r0.. of the
// row group (mamba2.py:84-89).
__device__ __forceinline__ void m2_conv_channel(const Mamba2PreP& p, int i, int r0, int nr, const long long* sslot) {
  constexpr int RM = kM2Rows;
  const int mi = p.mi, bc = p.bc;
  const bool isx = i < mi, isb = !isx && i < mi + bc;
  const int c = isx ? i : (isb ? i - mi : i - mi - bc), C = isx ? mi : bc;
  float* base = isx ? p.xconv : (isb ? p.bconv : p.cconv);
  const long long cs = isx ? p.xcs : (isb ? p.bcs : p.ccs);
  const float* w = isx ? p.wx : (isb ? p.wb : p.wc);
  const float* bias = isx ? p.bx : (isb ? p.bb : p.bcv);
  float* out = isx ? p.xs : (isb ? p.bs : p.cs);
  const int pi = isx ? i : mi + i;  // the proj row is [x | z | b | c]: b and c sit after z
  float s0[RM], s1[RM], s2[RM], xv[RM];
#pragma unroll
  for (int rr = 0; rr < RM; ++rr) {
    if (rr < nr) {
      const float* st = base + sslot[rr] * cs;
      s0[rr] = st[c];
      s1[rr] = st[C + c];
      s2[rr] = st[2 * C + c];
      xv[rr] = p.proj[size_t(r0 + rr) * p.ldp + pi];
    }
  }
  const float w0 = w[c], w1 = w[C + c], w2 = w[2 * C + c], w3 = w[3 * C + c], b0 = bias[c];
#pragma unroll
  for (int rr = 0; rr < RM; ++rr) {
    if (rr < nr) {
      // CausalConv1d over [state, x] (model/modules.py:37-41)
      float acc = w0 * s0[rr];
      acc = fmaf(w1, s1[rr], acc);
      acc = fmaf(w2, s2[rr], acc);
      acc = fmaf(w3, xv[rr], acc);
      float* st = base + sslot[rr] * cs;
      st[c] = s1[rr];
      st[C + c] = s2[rr];
      st[2 * C + c] = xv[rr];
      out[size_t(r0 + rr) * C + c] = siluf_(acc + b0);
    }
  }
}
// dt = softplus(dt_proj(t)); decay = exp(a * dt) (mamba2.py:81, 92-97) of head
// h by one warp for the row group: lanes stride the weight row, KC loads of it
// (and of each row's input) in flight before they are summed, in k order.
template <int KC>
__device__ __forceinline__ void m2_dt_head(const Mamba2PreP& p, int h, int r0, int nr, int lane) {
  constexpr int RM = kM2Rows;
  const float* w = p.dtw + size_t(h) * p.H;
  float acc[RM];
#pragma unroll
  for (int rr = 0; rr < RM; ++rr) acc[rr] = 0.f;
  for (int k0 = lane; k0 < p.H; k0 += 32 * KC) {
    float wv[KC], tv[RM][KC];
#pragma unroll
    for (int u = 0; u < KC; ++u) {
      const int k = k0 + 32 * u;
      wv[u] = k < p.H ? w[k] : 0.f;
#pragma unroll
      for (int rr = 0; rr < RM; ++rr) tv[rr][u] = (rr < nr && k < p.H) ? p.tin[size_t(r0 + rr) * p.H + k] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < KC; ++u) {
      if (k0 + 32 * u >= p.H) break;
#pragma unroll
      for (int rr = 0; rr < RM; ++rr)
        if (rr < nr) acc[rr] = fmaf(tv[rr][u], wv[u], acc[rr]);
    }
  }
#pragma unroll
  for (int rr = 0; rr < RM; ++rr) {
    const float v = warp_sum(acc[rr]);
    if (lane == 0 && rr < nr) {
      const float d = softplusf_(v + p.dtb[h]);
      p.dt[size_t(r0 + rr) * p.nh + h] = d;
      p.dc[size_t(r0 + rr) * p.nh + h] = expf(p.a[h] * d);
    }
  }
}
__global__ void __launch_bounds__(kRowThreads) k_mamba2_pre_rows(const Mamba2PreP p) {
  pdl_wait();
  constexpr int RM = kM2Rows;
  const int r0 = blockIdx.x * RM;
  const int nr = min(RM, live_rows(p.rc.n_dev, p.rc.rows) - r0);
  if (nr <= 0) return;
  __shared__ long long sslot[RM];
  if (threadIdx.x < nr) sslot[threadIdx.x] = row_slot(p.rc, r0 + threadIdx.x);
  __syncthreads();
  for (int i = threadIdx.x; i < p.mi + 2 * p.bc; i += blockDim.x) m2_conv_channel(p, i, r0, nr, sslot);
  const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int h = threadIdx.x >> 5; h < p.nh; h += nw) m2_dt_head<4>(p, h, r0, nr, lane);
}
// The same for steps of few rows, where one CTA per row group leaves most SMs
// idle: CTAs x < m2_conv_ctas convolve kRowThreads channels each, the rest
// compute dt for one head per warp; grid y = row groups.
constexpr int kM2SplitRows = 64;  // steps up to this many rows take k_mamba2_pre_split
__host__ __device__ inline int m2_conv_ctas(int mi, int bc) { return (mi + 2 * bc + kRowThreads - 1) / kRowThreads; }
__global__ void __launch_bounds__(kRowThreads) k_mamba2_pre_split(const Mamba2PreP p) {
  {
    const int ncv = m2_conv_ctas(p.mi, p.bc);
    if (int(blockIdx.x) >= ncv) {  // this CTA's dt_proj rows
      const int h0 = (blockIdx.x - ncv) * (kRowThreads / 32);
      const int nh = min(kRowThreads / 32, p.nh - h0);
      if (nh > 0) prefetch_l2(p.dtw + size_t(h0) * p.H, (long long)nh * p.H);
    }
  }
  pdl_wait();
  constexpr int RM = kM2Rows;
  const int r0 = blockIdx.y * RM;
  const int nr = min(RM, live_rows(p.rc.n_dev, p.rc.rows) - r0);
  if (nr <= 0) return;
  const int ncv = m2_conv_ctas(p.mi, p.bc);
  if (int(blockIdx.x) < ncv) {
    __shared__ long long sslot[RM];
    if (threadIdx.x < nr) sslot[threadIdx.x] = row_slot(p.rc, r0 + threadIdx.x);
    __syncthreads();
    const int i = blockIdx.x * kRowThreads + threadIdx.x;
    if (i < p.mi + 2 * p.bc) m2_conv_channel(p, i, r0, nr, sslot);
  } else {
    const int h = (blockIdx.x - ncv) * (kRowThreads / 32) + (threadIdx.x >> 5);
    if (h < p.nh) m2_dt_head<16>(p, h, r0, nr, threadIdx.x & 31);
  }
}

struct Mamba2PostP {
  RowCtx rc;
  const float* ys; const float* xs; const float* proj; int ldp; int mi, hs;
  const float* d; const float* nw; void* A; int at;
};
__global__ void __launch_bounds__(kRowThreads) k_mamba2_post(const Mamba2PostP p) {
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  extern __shared__ float g[];
  __shared__ float red[32];
  const float* y = p.ys + size_t(r) * p.mi;
  const float* x = p.xs + size_t(r) * p.mi;
  const float* z = p.proj + size_t(r) * p.ldp + p.mi;
  float ss = 0.f;
  for (int c = threadIdx.x; c < p.mi; c += blockDim.x) {
    // y = state_contrib + D*x; y *= silu(z) (mamba2.py:158-163)
    const float v = (y[c] + p.d[c / p.hs] * x[c]) * siluf_(z[c]);
    g[c] = v;
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / float(p.mi) + 1e-5f);  // RMSNorm eps 1e-5 (mamba2.py:45)
  for (int c = threadIdx.x; c < p.mi; c += blockDim.x) store_as(p.at, p.A, size_t(r) * p.mi + c, g[c] * inv * p.nw[c]);
}

// The same, one warp per row with 16-byte vectors (mi a multiple of 128 and
// hs of 4): RMSNorm's sum closes with shuffles, no shared memory or barrier.
constexpr int kM2PostRows = 8;
__global__ void __launch_bounds__(256) k_mamba2_post_w(const Mamba2PostP p) {
  pdl_wait();
  const int r = blockIdx.x * kM2PostRows + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (!row_live(p.rc, r)) return;
  const int n4 = p.mi >> 2;
  const float4* y = reinterpret_cast<const float4*>(p.ys + size_t(r) * p.mi);
  const float4* x = reinterpret_cast<const float4*>(p.xs + size_t(r) * p.mi);
  const float4* z = reinterpret_cast<const float4*>(p.proj + size_t(r) * p.ldp + p.mi);
  constexpr int V = 8;  // float4 per lane held in registers (mi <= 1024)
  float4 g[V];
  float ss = 0.f;
#pragma unroll
  for (int t = 0; t < V; ++t) {
    const int i = lane + 32 * t;
    if (i < n4) {
      const float4 yv = y[i], xv = x[i], zv = z[i];
      const float dh = p.d[(4 * i) / p.hs];  // the 4 columns share a head (hs % 4 == 0)
      // y = state_contrib + D*x; y *= silu(z) (mamba2.py:158-163)
      g[t].x = fmaf(dh, xv.x, yv.x) * siluf_(zv.x);
      g[t].y = fmaf(dh, xv.y, yv.y) * siluf_(zv.y);
      g[t].z = fmaf(dh, xv.z, yv.z) * siluf_(zv.z);
      g[t].w = fmaf(dh, xv.w, yv.w) * siluf_(zv.w);
      ss = fmaf(g[t].x, g[t].x, fmaf(g[t].y, g[t].y, fmaf(g[t].z, g[t].z, fmaf(g[t].w, g[t].w, ss))));
    }
  }
  ss = warp_sum(ss);
  const float inv = 1.0f / sqrtf(ss / float(p.mi) + 1e-5f);  // RMSNorm eps 1e-5 (mamba2.py:45)
  const float4* nw4 = reinterpret_cast<const float4*>(p.nw);
#pragma unroll
  for (int t = 0; t < V; ++t) {
    const int i = lane + 32 * t;
    if (i < n4) {
      const float4 w = nw4[i];
      const size_t o = size_t(r) * p.mi + 4 * size_t(i);
      store_as(p.at, p.A, o, g[t].x * inv * w.x);
      store_as(p.at, p.A, o + 1, g[t].y * inv * w.y);
      store_as(p.at, p.A, o + 2, g[t].z * inv * w.z);
      store_as(p.at, p.A, o + 3, g[t].w * inv * w.w);
    }
  }
}

class Mamba2Layer : public Layer {
 public:
  Mamba2Layer(const Dims& d, int lp) : d_(d), lp_(lp) {
    mi_ = d.mamba_inner(); nh_ = d.mamba_heads(); hs_ = d.m_hs; bc_ = d.m_bc; H_ = d.H;
    n1_ = 2 * mi_ + 2 * bc_;
  }
  void declare_state(StateArena& a) override {
    l_xc_ = a.add_conv(mi_, 3);
    l_bc_ = a.add_conv(bc_, 3);
    l_cc_ = a.add_conv(bc_, 3);
    l_ssm_ = a.add(nh_ * hs_ * bc_);
  }
  void load(WeightSource& s, WeightPack& w, const std::string& p) override {
    const long H = H_;
    o_w1_ = w.add_rows({{s.get(p + "input_proj.weight", mi_ * H), size_t(mi_ * H)},
                        {s.get(p + "z_proj.weight", mi_ * H), size_t(mi_ * H)},
                        {s.get(p + "b_proj.weight", bc_ * H), size_t(bc_ * H)},
                        {s.get(p + "c_proj.weight", bc_ * H), size_t(bc_ * H)}}, lp_);
    o_dtw_ = w.add(s.get(p + "dt_proj.weight", nh_ * H), nh_ * H, kF32);
    o_dtb_ = w.add(s.get(p + "dt_proj.bias", nh_), nh_, kF32);
    o_wx_ = w.add_conv(s.get(p + "input_conv.conv.weight", mi_ * 4), mi_, 4);
    o_bx_ = w.add(s.get(p + "input_conv.conv.bias", mi_), mi_, kF32);
    o_wb_ = w.add_conv(s.get(p + "b_conv.conv.weight", bc_ * 4), bc_, 4);
    o_bb_ = w.add(s.get(p + "b_conv.conv.bias", bc_), bc_, kF32);
    o_wc_ = w.add_conv(s.get(p + "c_conv.conv.weight", bc_ * 4), bc_, 4);
    o_bcv_ = w.add(s.get(p + "c_conv.conv.bias", bc_), bc_, kF32);
    o_a_ = w.add(s.get(p + "a", nh_), nh_, kF32);
    o_d_ = w.add(s.get(p + "d", nh_), nh_, kF32);
    o_nw_ = w.add(s.get(p + "norm.weight", mi_), mi_, kF32);
    o_out_ = w.add(s.get(p + "out_proj.weight", H * mi_), size_t(H) * mi_, lp_);
  }
  void resolve(const WeightPack& w, const StateArena& a) override {
    w1_ = w.ptr(o_w1_); dtw_ = w.ptr<float>(o_dtw_); dtb_ = w.ptr<float>(o_dtb_);
    wx_ = w.ptr<float>(o_wx_); bx_ = w.ptr<float>(o_bx_); wb_ = w.ptr<float>(o_wb_); bb_ = w.ptr<float>(o_bb_);
    wc_ = w.ptr<float>(o_wc_); bcv_ = w.ptr<float>(o_bcv_); a_ = w.ptr<float>(o_a_); dd_ = w.ptr<float>(o_d_);
    nw_ = w.ptr<float>(o_nw_); out_ = w.ptr(o_out_);
    xc_ = a.f32(l_xc_); bcs_ = a.f32(l_bc_); ccs_ = a.f32(l_cc_); ssm_ = a.f32(l_ssm_);
    sxc_ = a.stride(l_xc_); sbc_ = a.stride(l_bc_); scc_ = a.stride(l_cc_); sssm_ = a.stride(l_ssm_);
  }
  struct Buf { float *proj, *xs, *bs, *cs, *dt, *dc, *ys, *A; };
  Buf carve(uint8_t* base, int rows) const {
    Carver c{base};
    Buf b;
    b.proj = c.take<float>(size_t(rows) * n1_);
    b.xs = c.take<float>(size_t(rows) * mi_);
    b.bs = c.take<float>(size_t(rows) * bc_);
    b.cs = c.take<float>(size_t(rows) * bc_);
    b.dt = c.take<float>(size_t(rows) * nh_);
    b.dc = c.take<float>(size_t(rows) * nh_);
    b.ys = c.take<float>(size_t(rows) * mi_);
    b.A = c.take<float>(size_t(rows) * mi_);
    scratch_ = c.off;
    return b;
  }
  size_t scratch_bytes(int rows) const override {
    carve(nullptr, rows);
    return scratch_;
  }
  void forward(const StepCtx& c, const float* in, const void* in_lp, float* out, const float* residual,
               uint8_t* scratch, const RowEpi* post) override {
    const Buf b = carve(scratch, c.rows);
    const RowCtx rc{c.n_dev, c.rows, c.slots};
    const void* a1 = in_lp ? in_lp : in;
    const int a1t = in_lp ? lp_ : kF32;
    linear(c, a1, a1t, H_, w1_, lp_, nullptr, n1_, H_, b.proj, n1_);  // x, z, b, c (mamba2.py:77-80)
    Mamba2PreP pp{rc, b.proj, n1_, mi_, bc_, nh_, in, H_, dtw_, dtb_, xc_, sxc_, bcs_, sbc_, ccs_, scc_,
                  wx_, bx_, wb_, bb_, wc_, bcv_, a_, b.xs, b.bs, b.cs, b.dt, b.dc};
    if (c.rows <= kM2SplitRows) {
      const dim3 g(m2_conv_ctas(mi_, bc_) + ceil_div(nh_, kRowThreads / 32), ceil_div(c.rows, kM2Rows));
      launch_k(c.ln, k_mamba2_pre_split, g, dim3(kRowThreads), 0, c.s, pp);
    } else {
      launch_k(c.ln, k_mamba2_pre_rows, dim3(ceil_div(c.rows, kM2Rows)), dim3(kRowThreads), 0, c.s, pp);
    }
    SsmColsParams sp;
    sp.at = {ssm_, sssm_, c.slots, nullptr, c.rows, c.n_dev};
    sp.nh = nh_; sp.sh = hs_; sp.sc = bc_;
    sp.x = b.xs; sp.x_rs = mi_; sp.b = b.bs; sp.b_rs = bc_; sp.c = b.cs; sp.c_rs = bc_;
    sp.dt = b.dt; sp.dt_rs = nh_; sp.decay = b.dc; sp.dc_rs = nh_; sp.out = b.ys; sp.o_rs = mi_;
    sp.err = c.err;
    ssm_cols(sp, c.rows, c.s, c.ln_bulk);
    Mamba2PostP po{rc, b.ys, b.xs, b.proj, n1_, mi_, hs_, dd_, nw_, b.A, lp_};
    if (mi_ % 128 == 0 && mi_ <= 1024 && hs_ % 4 == 0 && n1_ % 4 == 0)
      launch_k(c.ln, k_mamba2_post_w, dim3(ceil_div(c.rows, kM2PostRows)), dim3(256), 0, c.s, po);
    else
      launch_k(c.ln, k_mamba2_post, dim3(c.rows), dim3(kRowThreads), mi_ * sizeof(float), c.s, po);
    linear(c, b.A, lp_, mi_, out_, lp_, nullptr, H_, mi_, out, H_, kActNone, residual, H_, nullptr, 0, post);  // out_proj (mamba2.py:165)
    B2E_CUDA(cudaGetLastError());
  }

  void latency_desc(LatLayer& L) const override {
    const void* w[] = {w1_, dtw_, dtb_, wx_, bx_, wb_, bb_, wc_, bcv_, a_, dd_, nw_, out_};
    for (size_t i = 0; i < sizeof(w) / sizeof(w[0]); ++i) L.w[i] = w[i];
    float* st[] = {xc_, bcs_, ccs_, ssm_};
    const long long ss[] = {sxc_, sbc_, scc_, sssm_};
    for (int i = 0; i < 4; ++i) { L.st[i] = st[i]; L.ss[i] = ss[i]; }
  }

 private:
  Dims d_;
  int lp_, mi_, nh_, hs_, bc_, H_, n1_;
  mutable size_t scratch_ = 0;
  int l_xc_ = 0, l_bc_ = 0, l_cc_ = 0, l_ssm_ = 0;
  size_t o_w1_, o_dtw_, o_dtb_, o_wx_, o_bx_, o_wb_, o_bb_, o_wc_, o_bcv_, o_a_, o_d_, o_nw_, o_out_;
  const void *w1_ = nullptr, *out_ = nullptr;
  const float *dtw_, *dtb_, *wx_, *bx_, *wb_, *bb_, *wc_, *bcv_, *a_, *dd_, *nw_;
  float *xc_, *bcs_, *ccs_, *ssm_;
  long long sxc_, sbc_, scc_, sssm_;
};

// ---------------------------------------------------------------- RetNet
// model/retnet.py:38-172.

struct RetPreP {
  RowCtx rc;
  const float* proj; int H, nh, hs;  // proj row: [q | k | v | g] (4H)
  int* pos; long long pos_s; float* scales; long long sc_s;
  const float* angle; const float* decay; float scaling;
  float* kr; float* qs;
};
__global__ void __launch_bounds__(kRowThreads) k_retnet_pre(const RetPreP p) {
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  const long long slot = row_slot(p.rc, r);
  const float* q = p.proj + size_t(r) * 4 * p.H;
  const float* k = q + p.H;
  int* pos = p.pos + slot * p.pos_s;
  float* sc = p.scales + slot * p.sc_s;
  const float fpos = float(*pos);  // int32 counter promoted to float32 (retnet.py:78)
  for (int e = threadIdx.x; e < p.H; e += blockDim.x) {
    const int n = e / p.hs, j = e - n * p.hs;
    const int mate = (j & 1) ? e - 1 : e + 1;
    const float arg = fpos * p.angle[j];
    const float s = sinf(arg), co = cosf(arg);
    // rotate_every_two: even j takes -x[j+1], odd j takes x[j-1] (retnet.py:9-13)
    const float qr = (j & 1) ? q[mate] : -q[mate];
    const float kk = k[e] * p.scaling, km = k[mate] * p.scaling;  // k *= hs^-1/2 (retnet.py:71)
    const float kr = (j & 1) ? km : -km;
    const float ns = sc[n] * p.decay[n] + 1.0f;  // scales*decay + 1 (retnet.py:93)
    const float f = 1.0f / sqrtf(ns);
    p.qs[size_t(r) * p.H + e] = (q[e] * co + qr * s) * f;  // q_rope * scale (retnet.py:81,94-101)
    p.kr[size_t(r) * p.H + e] = kk * co + kr * s;          // k_rope (retnet.py:82)
  }
  __syncthreads();  // every thread has read pos and scales
  for (int n = threadIdx.x; n < p.nh; n += blockDim.x) sc[n] = sc[n] * p.decay[n] + 1.0f;
  if (threadIdx.x == 0) *pos = *pos + 1;  // seq_offsets + 1 (retnet.py:172)
}

struct RetPostP {
  RowCtx rc;
  const float* o; const float* proj; int H, nh, hs; void* A; int at;
};
__global__ void __launch_bounds__(kRowThreads) k_retnet_post(const RetPostP p) {
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  extern __shared__ float inv[];  // per head
  const float* o = p.o + size_t(r) * p.H;
  const float* g = p.proj + size_t(r) * 4 * p.H + 3 * p.H;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int n = w; n < p.nh; n += nw) {  // per-head RMSNorm, eps 1e-6, no affine (retnet.py:33,168)
    float ss = 0.f;
    for (int j = lane; j < p.hs; j += 32) ss = fmaf(o[n * p.hs + j], o[n * p.hs + j], ss);
    ss = warp_sum(ss);
    if (lane == 0) inv[n] = 1.0f / sqrtf(ss / float(p.hs) + 1e-6f);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < p.H; e += blockDim.x)
    store_as(p.at, p.A, size_t(r) * p.H + e, siluf_(g[e]) * (o[e] * inv[e / p.hs]));  // silu(g) * out (retnet.py:169)
}

class RetNetLayer : public Layer {
 public:
  RetNetLayer(const Dims& d, int lp) : d_(d), lp_(lp), H_(d.H), nh_(d.heads), hs_(d.retnet_hs()) {}
  void declare_state(StateArena& a) override {
    l_pos_ = a.add(1, kLeafI32);
    l_sc_ = a.add(nh_);
    l_S_ = a.add(nh_ * hs_ * hs_);
  }
  void load(WeightSource& s, WeightPack& w, const std::string& p) override {
    const size_t HH = size_t(H_) * H_;
    o_w1_ = w.add_rows({{s.get(p + "q_proj.weight", HH), HH}, {s.get(p + "k_proj.weight", HH), HH},
                        {s.get(p + "v_proj.weight", HH), HH}, {s.get(p + "g_proj.weight", HH), HH}}, lp_);
    o_out_ = w.add(s.get(p + "out_proj.weight", HH), HH, lp_);
    o_decay_ = w.add(s.get(p + "decay", nh_), nh_, kF32);
    o_angle_ = w.add(s.get(p + "angle", hs_), hs_, kF32);
  }
  void resolve(const WeightPack& w, const StateArena& a) override {
    w1_ = w.ptr(o_w1_); out_ = w.ptr(o_out_); decay_ = w.ptr<float>(o_decay_); angle_ = w.ptr<float>(o_angle_);
    pos_ = a.i32(l_pos_); sc_ = a.f32(l_sc_); S_ = a.f32(l_S_);
    spos_ = a.stride(l_pos_); ssc_ = a.stride(l_sc_); sS_ = a.stride(l_S_);
  }
  struct Buf { float *proj, *kr, *qs, *o, *A; };
  Buf carve(uint8_t* base, int rows) const {
    Carver c{base};
    Buf b;
    b.proj = c.take<float>(size_t(rows) * 4 * H_);
    b.kr = c.take<float>(size_t(rows) * H_);
    b.qs = c.take<float>(size_t(rows) * H_);
    b.o = c.take<float>(size_t(rows) * H_);
    b.A = c.take<float>(size_t(rows) * H_);
    scratch_ = c.off;
    return b;
  }
  size_t scratch_bytes(int rows) const override {
    carve(nullptr, rows);
    return scratch_;
  }
  void forward(const StepCtx& c, const float* in, const void* in_lp, float* out, const float* residual,
               uint8_t* scratch, const RowEpi* post) override {
    const Buf b = carve(scratch, c.rows);
    const RowCtx rc{c.n_dev, c.rows, c.slots};
    linear(c, in_lp ? in_lp : in, in_lp ? lp_ : kF32, H_, w1_, lp_, nullptr, 4 * H_, H_, b.proj, 4 * H_);  // q, k, v, g (retnet.py:66-69)
    RetPreP pp{rc, b.proj, H_, nh_, hs_, pos_, spos_, sc_, ssc_, angle_, decay_,
               float(std::pow(double(hs_), -0.5)), b.kr, b.qs};
    launch_k(c.ln, k_retnet_pre, dim3(c.rows), dim3(kRowThreads), 0, c.s, pp);
    OuterRowsParams op;
    op.at = {S_, sS_, c.slots, nullptr, c.rows, c.n_dev};
    op.nh = nh_; op.sh = hs_; op.sk = hs_;
    op.f = decay_; op.f_rs = 0; op.f_hs = 1;
    op.kv = b.kr; op.k_rs = H_; op.v = b.proj + 2 * H_; op.v_rs = 4 * H_;
    op.q = b.qs; op.q_rs = H_; op.out = b.o; op.o_rs = H_;
    op.err = c.err;
    outer_rows(op, c.rows, c.s, c.ln_bulk);
    RetPostP po{rc, b.o, b.proj, H_, nh_, hs_, b.A, lp_};
    launch_k(c.ln, k_retnet_post, dim3(c.rows), dim3(kRowThreads), nh_ * sizeof(float), c.s, po);
    linear(c, b.A, lp_, H_, out_, lp_, nullptr, H_, H_, out, H_, kActNone, residual, H_, nullptr, 0, post);  // out_proj (retnet.py:170)
    B2E_CUDA(cudaGetLastError());
  }

  void latency_desc(LatLayer& L) const override {
    L.w[0] = w1_; L.w[1] = out_; L.w[2] = decay_; L.w[3] = angle_;
    L.st[0] = reinterpret_cast<float*>(pos_); L.ss[0] = spos_;
    L.st[1] = sc_; L.ss[1] = ssc_;
    L.st[2] = S_; L.ss[2] = sS_;
  }

 private:
  Dims d_;
  int lp_, H_, nh_, hs_;
  mutable size_t scratch_ = 0;
  int l_pos_ = 0, l_sc_ = 0, l_S_ = 0;
  size_t o_w1_, o_out_, o_decay_, o_angle_;
  const void *w1_ = nullptr, *out_ = nullptr;
  const float *decay_, *angle_;
  int* pos_;
  float *sc_, *S_;
  long long spos_, ssc_, sS_;
};

// ------------------------------------------------------------------ Hawk
// model/hawk.py:8-95.

struct HawkConvP {
  RowCtx rc;
  const float* proj; int H;  // proj row: [gate (H) | recurrent (H)]
  float* conv; long long cs; const float* w; const float* b; float* xc;
};
__global__ void __launch_bounds__(kRowThreads) k_hawk_conv(const HawkConvP p) {
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  float* st = p.conv + row_slot(p.rc, r) * p.cs;
  const float* x = p.proj + size_t(r) * 2 * p.H + p.H;
  for (int c = threadIdx.x; c < p.H; c += blockDim.x)
    p.xc[size_t(r) * p.H + c] = conv_step(p.w, p.b, st, p.H, c, x[c]);  // hawk.py:80
}

struct RglruP {
  RowCtx rc;
  const float* gates; const float* xc; const float* proj; int H;
  float* h; long long hs; const float* a; void* A; int at;
};
__global__ void __launch_bounds__(kRowThreads) k_rglru(const RglruP p) {
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  float* h = p.h + row_slot(p.rc, r) * p.hs;
  const float* gi = p.gates + size_t(r) * 2 * p.H;
  const float* gr = gi + p.H;
  const float* x = p.xc + size_t(r) * p.H;
  const float* gate = p.proj + size_t(r) * 2 * p.H;
  for (int c = threadIdx.x; c < p.H; c += blockDim.x) {
    const float it = sigmoidf_(gi[c]), rt = sigmoidf_(gr[c]);  // hawk.py:31-32
    const float at = powf(p.a[c], 8.0f * rt);                   // a ** (c * r), c = 8 (hawk.py:35)
    const float mult = sqrtf(1.0f - at * at);                   // hawk.py:36
    const float hn = h[c] * at + mult * (it * x[c]);            // hawk.py:37
    h[c] = hn;
    store_as(p.at, p.A, size_t(r) * p.H + c, geluf_(gate[c]) * hn);  // out_proj(gate * h) (hawk.py:77,83-84)
  }
}

class HawkLayer : public Layer {
 public:
  HawkLayer(const Dims& d, int lp) : d_(d), lp_(lp), H_(d.H), bs_(d.hawk_bs()) {}
  void declare_state(StateArena& a) override {
    l_conv_ = a.add_conv(H_, 3);
    l_h_ = a.add(H_);
  }
  void load(WeightSource& s, WeightPack& w, const std::string& p) override {
    const size_t HH = size_t(H_) * H_, BB = size_t(4) * bs_ * bs_;
    o_w1_ = w.add_rows({{s.get(p + "gate_proj.weight", HH), HH}, {s.get(p + "recurrent_proj.weight", HH), HH}}, lp_);
    o_cw_ = w.add_conv(s.get(p + "conv.conv.weight", H_ * 4), H_, 4);
    o_cb_ = w.add(s.get(p + "conv.conv.bias", H_), H_, kF32);
    o_a_ = w.add(s.get(p + "rglru.a", H_), H_, kF32);
    o_gw_ = w.add_rows({{s.get(p + "rglru.input_gate.weight", BB), BB},
                        {s.get(p + "rglru.recurrence_gate.weight", BB), BB}}, kF32);
    o_out_ = w.add(s.get(p + "out_proj.weight", HH), HH, lp_);
  }
  void resolve(const WeightPack& w, const StateArena& a) override {
    w1_ = w.ptr(o_w1_); out_ = w.ptr(o_out_); cw_ = w.ptr<float>(o_cw_); cb_ = w.ptr<float>(o_cb_);
    a_ = w.ptr<float>(o_a_); gw_ = w.ptr<float>(o_gw_);
    conv_ = a.f32(l_conv_); h_ = a.f32(l_h_); sconv_ = a.stride(l_conv_); sh_ = a.stride(l_h_);
  }
  struct Buf { float *proj, *xc, *gates, *A; };
  Buf carve(uint8_t* base, int rows) const {
    Carver c{base};
    Buf b;
    b.proj = c.take<float>(size_t(rows) * 2 * H_);
    b.xc = c.take<float>(size_t(rows) * H_);
    b.gates = c.take<float>(size_t(rows) * 2 * H_);
    b.A = c.take<float>(size_t(rows) * H_);
    scratch_ = c.off;
    return b;
  }
  size_t scratch_bytes(int rows) const override {
    carve(nullptr, rows);
    return scratch_;
  }
  void forward(const StepCtx& c, const float* in, const void* in_lp, float* out, const float* residual,
               uint8_t* scratch, const RowEpi* post) override {
    const Buf b = carve(scratch, c.rows);
    const RowCtx rc{c.n_dev, c.rows, c.slots};
    linear(c, in_lp ? in_lp : in, in_lp ? lp_ : kF32, H_, w1_, lp_, nullptr, 2 * H_, H_, b.proj, 2 * H_);  // gate_proj, recurrent_proj (hawk.py:77-78)
    HawkConvP cp{rc, b.proj, H_, conv_, sconv_, cw_, cb_, b.xc};
    launch_k(c.ln, k_hawk_conv, dim3(c.rows), dim3(kRowThreads), 0, c.s, cp);
    // RG-LRU gates: two BlockLinears of 4 diagonal blocks, fp32 (hawk.py:31-32, modules.py:71-79)
    GemmParams g;
    g.groups = 8;
    for (int s = 0; s < 2; ++s)
      for (int j = 0; j < 4; ++j) {
        GemmGroup& gg = g.g[s * 4 + j];
        gg.A = b.xc + j * bs_;
        gg.W = gw_ + (size_t(s) * 4 + j) * bs_ * bs_;
        gg.C = b.gates + s * H_ + j * bs_;
      }
    g.M_max = c.rows; g.M_dev = c.n_dev; g.N = bs_; g.K = bs_;
    g.lda = H_; g.ldw = bs_; g.ldc = 2 * H_;
    gemm(g, c.s);
    RglruP rp{rc, b.gates, b.xc, b.proj, H_, h_, sh_, a_, b.A, lp_};
    launch_k(c.ln, k_rglru, dim3(c.rows), dim3(kRowThreads), 0, c.s, rp);
    linear(c, b.A, lp_, H_, out_, lp_, nullptr, H_, H_, out, H_, kActNone, residual, H_, nullptr, 0, post);  // out_proj (hawk.py:84)
    B2E_CUDA(cudaGetLastError());
  }

  void latency_desc(LatLayer& L) const override {
    L.w[0] = w1_; L.w[1] = cw_; L.w[2] = cb_; L.w[3] = a_; L.w[4] = gw_; L.w[5] = out_;
    L.st[0] = conv_; L.ss[0] = sconv_;
    L.st[1] = h_; L.ss[1] = sh_;
  }

 private:
  Dims d_;
  int lp_, H_, bs_;
  mutable size_t scratch_ = 0;
  int l_conv_ = 0, l_h_ = 0;
  size_t o_w1_, o_cw_, o_cb_, o_a_, o_gw_, o_out_;
  const void *w1_ = nullptr, *out_ = nullptr;
  const float *cw_, *cb_, *a_, *gw_;
  float *conv_, *h_;
  long long sconv_, sh_;
};

// ----------------------------------------------------------------- xLSTM
// model/xlstm.py:21-379: sLSTM block, then mLSTM block, then LayerNorm.

struct SlstmPreP {
  RowCtx rc;
  const float* t; int H, nbl, bs;
  const float* lnw;
  float* conv; long long cs; const float* cw; const float* cb;
  const float* h; long long hst;
  float* axc; float* axn;  // [row][2H]: per block j, [input_j | h_j]
};
__global__ void __launch_bounds__(kRowThreads) k_slstm_pre(const SlstmPreP p) {
  prefetch_l1(p.lnw, p.H);
  prefetch_l1(p.cw, 4 * p.H);
  prefetch_l1(p.cb, p.H);
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  extern __shared__ float xn[];
  __shared__ float gm[1], gr[1];
  const long long slot = row_slot(p.rc, r);
  const float* t = p.t + size_t(r) * p.H;
  for (int c = threadIdx.x; c < p.H; c += blockDim.x) xn[c] = t[c];
  __syncthreads();
  group_stats(xn, 1, p.H, 1e-5f, gm, gr);  // LayerNorm(bias=False) (xlstm.py:287,307)
  const float mu = gm[0], rs = gr[0];
  float* st = p.conv + slot * p.cs;
  const float* h = p.h + slot * p.hst;
  float* axc = p.axc + size_t(r) * 2 * p.H;
  float* axn = p.axn + size_t(r) * 2 * p.H;
  const int H = p.H;
  for (int c0 = threadIdx.x; c0 < H; c0 += kEU * blockDim.x) {
    float tv[kEU], lw[kEU], s0[kEU], s1[kEU], s2[kEU], hv[kEU], w0[kEU], w1[kEU], w2[kEU], w3[kEU], cb[kEU];
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int c = c0 + u * blockDim.x;
      if (c < H) {
        tv[u] = t[c]; lw[u] = p.lnw[c]; hv[u] = h[c];
        s0[u] = st[c]; s1[u] = st[H + c]; s2[u] = st[2 * H + c];
        w0[u] = p.cw[c]; w1[u] = p.cw[H + c]; w2[u] = p.cw[2 * H + c]; w3[u] = p.cw[3 * H + c]; cb[u] = p.cb[c];
      }
    }
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int c = c0 + u * blockDim.x;
      if (c >= H) break;
      const float x = (tv[u] - mu) * rs * lw[u];
      // CausalConv1d over [state, x] (model/modules.py:37-41) + SiLU (xlstm.py:309-310)
      float acc = w0[u] * s0[u];
      acc = fmaf(w1[u], s1[u], acc);
      acc = fmaf(w2[u], s2[u], acc);
      acc = fmaf(w3[u], x, acc);
      st[c] = s1[u];
      st[H + c] = s2[u];
      st[2 * H + c] = x;
      const float xc = siluf_(acc + cb[u]);
      const int j = c / p.bs, e = c - j * p.bs;
      axc[j * 2 * p.bs + e] = xc;
      axn[j * 2 * p.bs + e] = x;
      axc[j * 2 * p.bs + p.bs + e] = hv[u];
      axn[j * 2 * p.bs + p.bs + e] = hv[u];
    }
  }
}

struct SlstmPostP {
  RowCtx rc;
  const float* G; const float* t; int H, nbl;  // G row: [i | f | z | o] (4H), pre-activations
  float *hs_, *cs_, *ns_, *ms_; long long h_s, c_s, n_s, m_s;
  const float *gnw, *gnb, *mlnw;
  float* x1; void* xn2; int at;
};
__global__ void __launch_bounds__(kRowThreads) k_slstm_post(const SlstmPostP p) {
  prefetch_l1(p.gnw, p.H);
  prefetch_l1(p.gnb, p.H);
  prefetch_l1(p.mlnw, p.H);
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  extern __shared__ float sm[];
  float* y = sm;          // H
  float* x1 = sm + p.H;   // H
  __shared__ float gm[64], gr[64];
  const long long slot = row_slot(p.rc, r);
  const float* G = p.G + size_t(r) * 4 * p.H;
  float* hh = p.hs_ + slot * p.h_s;
  float* cc = p.cs_ + slot * p.c_s;
  float* nn = p.ns_ + slot * p.n_s;
  float* mm = p.ms_ + slot * p.m_s;
  const int H = p.H;
  for (int e0 = threadIdx.x; e0 < H; e0 += kEU * blockDim.x) {
    float gi[kEU], gf[kEU], gz[kEU], go[kEU], mo[kEU], co[kEU], no[kEU];
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e < H) {
        gi[u] = G[e]; gf[u] = G[H + e]; gz[u] = G[2 * H + e]; go[u] = G[3 * H + e];
        mo[u] = mm[e]; co[u] = cc[e]; no[u] = nn[e];
      }
    }
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e >= H) break;
      // SLSTMCell.forward (xlstm.py:247-262)
      const float lfm = mo[u] + logsigmoidf_(gf[u]);
      const float mn = fmaxf(gi[u], lfm);
      const float og = sigmoidf_(go[u]);
      const float ig = expf(gi[u] - mn);
      const float fg = expf(lfm - mn);
      const float cn = fg * co[u] + ig * tanhf(gz[u]);
      const float nv = fg * no[u] + ig;
      const float yv = og * cn / (nv + 1e-6f);
      cc[e] = cn; nn[e] = nv; mm[e] = mn; hh[e] = yv;
      y[e] = yv;
    }
  }
  __syncthreads();
  group_stats(y, p.nbl, H / p.nbl, 1e-5f, gm, gr);  // GroupNorm(num_heads) (xlstm.py:300,316)
  const float* t = p.t + size_t(r) * H;
  const int gs = H / p.nbl;
  for (int e0 = threadIdx.x; e0 < H; e0 += kEU * blockDim.x) {
    float gw[kEU], gb[kEU], tv[kEU];
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e < H) { gw[u] = p.gnw[e]; gb[u] = p.gnb[e]; tv[u] = t[e]; }
    }
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e >= H) break;
      const int g = e / gs;
      const float v = (y[e] - gm[g]) * gr[g] * gw[u] + gb[u] + tv[u];  // + skip (xlstm.py:318)
      x1[e] = v;
      p.x1[size_t(r) * H + e] = v;
    }
  }
  __syncthreads();
  group_stats(x1, 1, H, 1e-5f, gm, gr);  // mLSTM block LayerNorm (xlstm.py:182,202)
  for (int e0 = threadIdx.x; e0 < H; e0 += kEU * blockDim.x) {
    float mw[kEU];
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e < H) mw[u] = p.mlnw[e];
    }
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e >= H) break;
      store_as(p.at, p.xn2, size_t(r) * H + e, (x1[e] - gm[0]) * gr[0] * mw[u]);
    }
  }
}

// The whole sLSTM block for kSlRows rows per CTA (xlstm.py:239-318) and the
// mLSTM block's input LayerNorm (xlstm.py:182,202): LayerNorm, conv + SiLU, the
// eight fp32 BlockLinears (i, f from the conv branch, z, o from the normed
// input, each plus a BlockLinear of the old h), the stabilized cell, GroupNorm
// and skip. One thread per hidden unit u holds the four gates of u for every
// row of the CTA; the weights are packed k-major ([2bs][4][H]) so a warp's 32
// units read 128 contiguous bytes per gate and k, shared by the CTA's rows.
constexpr int kSlRows = 16;
// Rows per CTA at hidden <= 128, where a CTA is only H/32 <= 4 warps: more CTAs
// of fewer rows keep more warps resident for the kernel's latency-bound phases.
constexpr int kSlRowsNarrow = 8;
// SLSTMCell.forward for one unit of one row (xlstm.py:247-262): gates i, f, z, o
// in, (c, n, m) updated in place, h out. Out of line, so that the rows of a
// k_slstm_fused CTA share one copy of the transcendental code.
__device__ __noinline__ float slstm_cell(float i, float f, float z, float o, float& c, float& n, float& m) {
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
constexpr int kSlMaxGroups = 16;  // sLSTM heads (GroupNorm groups) per row
// The gate loop's operands in shared memory: rows 2q and 2q+1 of unit k side by
// side, so one 64-bit load is the operand pair of an fma.rn.f32x2.
__device__ __forceinline__ int sl_pair(int r, int k, int H) { return (((r >> 1) * H + k) << 1) + (r & 1); }
__device__ __forceinline__ unsigned long long f32x2(float lo, float hi) {
  unsigned long long v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  return v;
}
__device__ __forceinline__ float2 f32x2_split(unsigned long long v) {
  float2 f;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(v));
  return f;
}
// d = a * b + d on both halves, each rounded as fmaf rounds it
__device__ __forceinline__ void fma_f32x2(unsigned long long& d, unsigned long long a, unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(d) : "l"(a), "l"(b));
}
constexpr size_t kSlSmemMax = 96 * 1024;
struct SlstmFusedP {
  RowCtx rc;
  const float* t; int H, nbl, bs;
  const float* lnw;
  float* conv; long long cs; const float* cw; const float* cb;
  float *hs_, *cs_, *ns_, *ms_; long long h_s, c_s, n_s, m_s;
  const float* wt;    // [2bs][4][H]: k (input half, then state half), gate i f z o, unit
  const float* bias;  // [4][H]
  const float *gnw, *gnb, *mlnw;
  float* x1; void* xn2; int at;
};
// HT: the hidden size when fixed at compile time (shared-memory row offsets
// and weight strides become immediates), else 0.
template <int RB, int HT>
__global__ void __launch_bounds__(512) k_slstm_fused(const SlstmFusedP p) {
  pdl_wait();
  const int r0 = blockIdx.x * RB;
  const int nr = min(RB, live_rows(p.rc.n_dev, p.rc.rows) - r0);
  if (nr <= 0) return;
  extern __shared__ float4 sl_raw[];
  const int H = HT ? HT : p.H, u = threadIdx.x;  // blockDim.x == H
  // three planes of RB x H floats: row-major [RB][H], except in the gate loop,
  // whose operands are stored pair-interleaved (sl_pair)
  float* xc = reinterpret_cast<float*>(sl_raw);  // conv+SiLU branch (pairs), later the cell output y
  float* xn = xc + RB * H;                       // input, then LayerNorm(input) (pairs), later x1
  float* hb = xn + RB * H;                       // old h (pairs)
  __shared__ float gm[RB * kSlMaxGroups], gr[RB * kSlMaxGroups];
  __shared__ long long slot[RB];
  if (u < RB) slot[u] = u < nr ? row_slot(p.rc, r0 + u) : 0;
#pragma unroll
  for (int r = 0; r < RB; ++r) xn[r * H + u] = r < nr ? p.t[size_t(r0 + r) * H + u] : 0.f;
  __syncthreads();
  group_stats(xn, RB, H, 1e-5f, gm, gr);  // LayerNorm(bias=False) per row (xlstm.py:287,307)
  {
    // every row's conv taps and h first, then the updates
    float s0[RB], s1[RB], s2[RB], ho[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      if (r < nr) {
        const float* st = p.conv + slot[r] * p.cs;
        s0[r] = st[u];
        s1[r] = st[H + u];
        s2[r] = st[2 * H + u];
        ho[r] = p.hs_[slot[r] * p.h_s + u];
      } else {
        s0[r] = s1[r] = s2[r] = ho[r] = 0.f;
      }
    }
    const float w0 = p.cw[u], w1 = p.cw[H + u], w2 = p.cw[2 * H + u], w3 = p.cw[3 * H + u], cb = p.cb[u], lw = p.lnw[u];
    float xv[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) xv[r] = (xn[r * H + u] - gm[r]) * gr[r] * lw;
    __syncthreads();  // every row-major input read before the pair-interleaved writes
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const float x = xv[r];
      // CausalConv1d over [state, x] (model/modules.py:37-41) and SiLU (xlstm.py:309-310)
      float acc = w0 * s0[r];
      acc = fmaf(w1, s1[r], acc);
      acc = fmaf(w2, s2[r], acc);
      acc = fmaf(w3, x, acc);
      const int ip = sl_pair(r, u, H);
      xc[ip] = r < nr ? siluf_(acc + cb) : 0.f;
      xn[ip] = x;
      hb[ip] = ho[r];
      if (r < nr) {
        float* st = p.conv + slot[r] * p.cs;
        st[u] = s1[r];
        st[H + u] = s2[r];
        st[2 * H + u] = x;
      }
    }
  }
  __syncthreads();
  // gates: acc[g][r] = sum_k W_g[u][k] * a_g[r][k] over k < bs (input half:
  // the conv branch for i, f, the normed input for z, o) and bs <= k < 2bs
  // (the old h of u's block, all gates) (xlstm.py:250-253, 312-315). Rows 2q
  // and 2q+1 of a gate are one f32x2 pair, updated by one fma.rn.f32x2 in the
  // same order of k as one fmaf per row.
  const int bs = p.bs, j0 = (u / bs) * bs;
  unsigned long long acc2[4][RB / 2];
#pragma unroll
  for (int g = 0; g < 4; ++g)
#pragma unroll
    for (int q = 0; q < RB / 2; ++q) acc2[g][q] = 0ull;  // (+0.f, +0.f)
  const float* wt = p.wt + u;
  const size_t kst = size_t(4) * H;  // one k of the packed weights
  for (int half = 0; half < 2; ++half) {
    const unsigned long long* a0 = reinterpret_cast<const unsigned long long*>(half ? hb : xc) + j0;
    const unsigned long long* a1 = reinterpret_cast<const unsigned long long*>(half ? hb : xn) + j0;
    const float* wk = wt + size_t(half) * bs * kst;
    for (int k = 0; k < bs; k += 4) {
      float w[4][4];  // [kk][gate]
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int g = 0; g < 4; ++g) w[kk][g] = __ldg(wk + (k + kk) * kst + size_t(g) * H);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const unsigned long long wi = f32x2(w[kk][0], w[kk][0]), wf = f32x2(w[kk][1], w[kk][1]);
        const unsigned long long wz = f32x2(w[kk][2], w[kk][2]), wo = f32x2(w[kk][3], w[kk][3]);
#pragma unroll
        for (int q = 0; q < RB / 2; ++q) {
          const unsigned long long a = a0[size_t(q) * H + k + kk], b = a1[size_t(q) * H + k + kk];
          fma_f32x2(acc2[0][q], a, wi);
          fma_f32x2(acc2[1][q], a, wf);
          fma_f32x2(acc2[2][q], b, wz);
          fma_f32x2(acc2[3][q], b, wo);
        }
      }
    }
  }
  __syncthreads();  // xc, xn, hb are free
  {
    const float bi = p.bias[u], bf = p.bias[H + u], bz = p.bias[2 * H + u], bo = p.bias[3 * H + u];
    constexpr int RC = RB < 8 ? RB : 8;  // rows whose state loads are in flight together
#pragma unroll
    for (int rc = 0; rc < RB; rc += RC) {
      float co[RC], no[RC], mo[RC];
#pragma unroll
      for (int q = 0; q < RC; ++q) {
        const int r = rc + q;
        const bool on = r < nr;
        co[q] = on ? p.cs_[slot[r] * p.c_s + u] : 0.f;
        no[q] = on ? p.ns_[slot[r] * p.n_s + u] : 0.f;
        mo[q] = on ? p.ms_[slot[r] * p.m_s + u] : 0.f;
      }
#pragma unroll
      for (int q = 0; q < RC; ++q) {
        const int r = rc + q;
        float cn = co[q], nv = no[q], mn = mo[q];
        const float2 gi = f32x2_split(acc2[0][r >> 1]), gf = f32x2_split(acc2[1][r >> 1]);
        const float2 gz = f32x2_split(acc2[2][r >> 1]), go = f32x2_split(acc2[3][r >> 1]);
        const bool odd = r & 1;
        const float yv = slstm_cell((odd ? gi.y : gi.x) + bi, (odd ? gf.y : gf.x) + bf, (odd ? gz.y : gz.x) + bz,
                                    (odd ? go.y : go.x) + bo, cn, nv, mn);
        xc[r * H + u] = yv;
        if (r < nr) {
          p.cs_[slot[r] * p.c_s + u] = cn;
          p.ns_[slot[r] * p.n_s + u] = nv;
          p.ms_[slot[r] * p.m_s + u] = mn;
          p.hs_[slot[r] * p.h_s + u] = yv;
        }
      }
    }
  }
  __syncthreads();
  const int gs = H / p.nbl, gu = u / gs;
  group_stats(xc, RB * p.nbl, gs, 1e-5f, gm, gr);  // GroupNorm(num_heads) per row (xlstm.py:300,316)
  {
    const float gw = p.gnw[u], gb = p.gnb[u];
    float tv[RB];  // every row's skip input loaded before the first store below
#pragma unroll
    for (int r = 0; r < RB; ++r) tv[r] = r < nr ? p.t[size_t(r0 + r) * H + u] : 0.f;
#pragma unroll
    for (int r = 0; r < RB; ++r) {
      const float t = tv[r];
      const float v = (xc[r * H + u] - gm[r * p.nbl + gu]) * gr[r * p.nbl + gu] * gw + gb + t;  // + skip (xlstm.py:318)
      xn[r * H + u] = v;
      if (r < nr) p.x1[size_t(r0 + r) * H + u] = v;
    }
  }
  __syncthreads();
  group_stats(xn, RB, H, 1e-5f, gm, gr);  // mLSTM block LayerNorm (xlstm.py:182,202)
  const float mw = p.mlnw[u];
#pragma unroll
  for (int r = 0; r < RB; ++r)
    if (r < nr) store_as(p.at, p.xn2, size_t(r0 + r) * H + u, (xn[r * H + u] - gm[r]) * gr[r] * mw);
}

// The mLSTM block between x_proj/gate_proj and the cell's state update, for
// kMidRows rows per CTA (xlstm.py:92-132, 198-213): conv1d + SiLU, the q/k/v
// BlockLinears (4x4 blocks), the input/forget gate projections over cat(q,k,v)
// (fp32, weights shared by the CTA's rows through L1), the stabilized gates and
// the normalizer state. Outputs: xca (conv+SiLU), q | k/sqrt(hs) | v, (i, f)
// gate values and the h-denominator per head; the conv, n and m leaves updated.
struct MlstmMidP {
  RowCtx rc;
  const float* proj; int mi, nh, hs;          // proj row: [x_mlstm (mi) | x_gate (mi)]
  float* conv; long long cs; const float* cw; const float* cb;
  const float *wq, *wk, *wv;                  // (mi/4, 4, 4)
  const float* gw; const float* gb;           // [2nh][3mi] (igate rows, then fgate rows), [2nh]
  float* n; long long n_s; float* m; long long m_s;
  float* xca; float* qkv; float* g2; float* den;  // [row][mi], [row][3mi], [row][2nh] (i | f), [row][nh]
  int rows_per_cta;
};
__global__ void __launch_bounds__(kRowThreads, 3) k_mlstm_mid(const MlstmMidP p) {
  pdl_wait();
  const int r0 = blockIdx.x * p.rows_per_cta;
  const int nr = min(p.rows_per_cta, live_rows(p.rc.n_dev, p.rc.rows) - r0);
  if (nr <= 0) return;
  extern __shared__ float smid[];  // [rows][3mi] q | k | v (k unscaled), [rows][mi] conv+SiLU, [rows][2nh] gate pre-activations
  constexpr int RM = 4, U = 6;     // rows per CTA at most; gate-weight vectors per lane at a time
  const int mi = p.mi, nh = p.nh, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  float* xcs = smid + size_t(p.rows_per_cta) * 3 * mi;
  float* gpre = xcs + size_t(p.rows_per_cta) * mi;
  __shared__ long long sslot[RM];
  if (tid < nr) sslot[tid] = row_slot(p.rc, r0 + tid);
  __syncthreads();
  // conv1d + SiLU (xlstm.py:206-207), consecutive channels on consecutive
  // lanes; every row's taps and input are loaded before any is updated
  for (int c = tid; c < mi; c += blockDim.x) {
    float s0[RM], s1[RM], s2[RM], xv[RM];
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      if (rr < nr) {
        const float* st = p.conv + sslot[rr] * p.cs;
        s0[rr] = st[c];
        s1[rr] = st[mi + c];
        s2[rr] = st[2 * mi + c];
        xv[rr] = p.proj[size_t(r0 + rr) * 2 * mi + c];
      }
    }
    const float w0 = p.cw[c], w1 = p.cw[mi + c], w2 = p.cw[2 * mi + c], w3 = p.cw[3 * mi + c], cb = p.cb[c];
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      if (rr < nr) {
        // CausalConv1d over [state, x] (model/modules.py:37-41)
        float acc = w0 * s0[rr];
        acc = fmaf(w1, s1[rr], acc);
        acc = fmaf(w2, s2[rr], acc);
        acc = fmaf(w3, xv[rr], acc);
        float* st = p.conv + sslot[rr] * p.cs;
        st[c] = s1[rr];
        st[mi + c] = s2[rr];
        st[2 * mi + c] = xv[rr];
        const float v = siluf_(acc + cb);
        xcs[rr * mi + c] = v;
        p.xca[size_t(r0 + rr) * mi + c] = v;
      }
    }
  }
  __syncthreads();
  // q/k from the conv branch, v from x_mlstm: BlockLinear with 4x4 blocks,
  // out[4b+kk] = sum_h x[4b+h] * W[b][kk][h] (xlstm.py:209-211); one output per
  // thread, its weight row W[b][kk][:] one 16-byte load shared by the CTA's rows
  for (int e = tid; e < mi; e += blockDim.x) {
    const float4 wq = __ldg(reinterpret_cast<const float4*>(p.wq) + e);
    const float4 wk = __ldg(reinterpret_cast<const float4*>(p.wk) + e);
    const float4 wv = __ldg(reinterpret_cast<const float4*>(p.wv) + e);
    float4 x0[RM];
#pragma unroll
    for (int rr = 0; rr < RM; ++rr)
      if (rr < nr) x0[rr] = reinterpret_cast<const float4*>(p.proj + size_t(r0 + rr) * 2 * mi)[e >> 2];
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      if (rr < nr) {
        const int r = r0 + rr;
        const float4 xc = reinterpret_cast<const float4*>(xcs + rr * mi)[e >> 2];
        const float aq = fmaf(xc.w, wq.w, fmaf(xc.z, wq.z, fmaf(xc.y, wq.y, xc.x * wq.x)));
        const float ak = fmaf(xc.w, wk.w, fmaf(xc.z, wk.z, fmaf(xc.y, wk.y, xc.x * wk.x)));
        const float av = fmaf(x0[rr].w, wv.w, fmaf(x0[rr].z, wv.z, fmaf(x0[rr].y, wv.y, x0[rr].x * wv.x)));
        float* q = smid + size_t(rr) * 3 * mi;
        q[e] = aq;
        q[mi + e] = ak;
        q[2 * mi + e] = av;
        p.qkv[size_t(r) * 3 * mi + e] = aq;
        p.qkv[size_t(r) * 3 * mi + 2 * mi + e] = av;
      }
    }
  }
  __syncthreads();
  // igate / fgate projections of cat(q, k, v) (xlstm.py:119-120): one warp per
  // head, its igate and fgate weight rows in registers (UG vectors each per lane
  // at a time), so each q/k/v vector read from shared memory feeds both gates,
  // against every row of the CTA
  constexpr int UG = U / 2;
  const int k4n = (3 * mi) >> 2;
  for (int h = warp; h < nh; h += nw) {
    const float4* wi4 = reinterpret_cast<const float4*>(p.gw + size_t(h) * 3 * mi);
    const float4* wf4 = reinterpret_cast<const float4*>(p.gw + size_t(nh + h) * 3 * mi);
    float ai[RM] = {0.f, 0.f, 0.f, 0.f}, af[RM] = {0.f, 0.f, 0.f, 0.f};
    for (int k0 = lane; k0 < k4n; k0 += 32 * UG) {
      float4 wi[UG], wf[UG];
#pragma unroll
      for (int u = 0; u < UG; ++u) {
        const bool in = k0 + 32 * u < k4n;
        wi[u] = in ? __ldg(wi4 + k0 + 32 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
        wf[u] = in ? __ldg(wf4 + k0 + 32 * u) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int rr = 0; rr < RM; ++rr) {
        if (rr >= nr) break;
        const float4* a = reinterpret_cast<const float4*>(smid + size_t(rr) * 3 * mi);
#pragma unroll
        for (int u = 0; u < UG; ++u) {
          if (k0 + 32 * u >= k4n) break;
          const float4 x = a[k0 + 32 * u];
          ai[rr] = fmaf(x.w, wi[u].w, fmaf(x.z, wi[u].z, fmaf(x.y, wi[u].y, fmaf(x.x, wi[u].x, ai[rr]))));
          af[rr] = fmaf(x.w, wf[u].w, fmaf(x.z, wf[u].z, fmaf(x.y, wf[u].y, fmaf(x.x, wf[u].x, af[rr]))));
        }
      }
    }
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      const float vi = warp_sum(ai[rr]), vf = warp_sum(af[rr]);
      if (lane == 0 && rr < nr) {
        gpre[rr * 2 * nh + h] = vi + p.gb[h];
        gpre[rr * 2 * nh + nh + h] = vf + p.gb[nh + h];
      }
    }
  }
  __syncthreads();
  // MLSTMCell gates and normalizer (xlstm.py:92-103, 121-132): one warp per head,
  // every row's state loads issued together
  const float sq = sqrtf(float(p.hs));
  for (int h = warp; h < nh; h += nw) {
    long long slot[RM];
    float mn[RM], i_g[RM], f_g[RM], qn[RM];
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      slot[rr] = rr < nr ? sslot[rr] : 0;
      mn[rr] = rr < nr ? p.m[slot[rr] * p.m_s + h] : 0.f;  // old m, replaced below
    }
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      const float ig = rr < nr ? gpre[rr * 2 * nh + h] : 0.f, fg = rr < nr ? gpre[rr * 2 * nh + nh + h] : 0.f;
      const float lf = logsigmoidf_(fg), mo = mn[rr];
      mn[rr] = fmaxf(ig, mo + lf);
      i_g[rr] = expf(ig - mn[rr]);
      f_g[rr] = expf(lf + mo - mn[rr]);
      qn[rr] = 0.f;
    }
    for (int j0 = 0; j0 < p.hs; j0 += 128) {
      float nold[RM][4];
#pragma unroll
      for (int rr = 0; rr < RM; ++rr)
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int j = j0 + lane + 32 * t;
          nold[rr][t] = (rr < nr && j < p.hs) ? p.n[slot[rr] * p.n_s + h * p.hs + j] : 0.f;
        }
#pragma unroll
      for (int rr = 0; rr < RM; ++rr) {
        if (rr >= nr) break;
        const float* q = smid + size_t(rr) * 3 * mi;
        float* nst = p.n + slot[rr] * p.n_s;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int j = j0 + lane + 32 * t;
          if (j >= p.hs) break;
          const int e = h * p.hs + j;
          const float ks = q[mi + e] / sq;  // k / sqrt(head_size) (xlstm.py:99)
          const float nv = f_g[rr] * nold[rr][t] + i_g[rr] * ks;
          p.qkv[size_t(r0 + rr) * 3 * mi + mi + e] = ks;
          nst[e] = nv;
          qn[rr] = fmaf(q[e], nv, qn[rr]);
        }
      }
    }
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      const float v = warp_sum(qn[rr]);
      if (lane == 0 && rr < nr) {
        const int r = r0 + rr;
        p.m[slot[rr] * p.m_s + h] = mn[rr];
        p.g2[size_t(r) * 2 * nh + h] = i_g[rr];
        p.g2[size_t(r) * 2 * nh + nh + h] = f_g[rr];
        p.den[size_t(r) * nh + h] = fmaxf(fabsf(v), expf(-mn[rr])) + 1e-6f;  // xlstm.py:130-132
      }
    }
  }
}

constexpr size_t kMidSmemMax = 96 * 1024;
// Rows per k_mlstm_mid CTA: up to 4, within kMidSmemMax of shared memory.
// k_mlstm_mid for steps of a few rows, where one CTA per four rows leaves most
// SMs idle (one request at the default dims: 56 us on one SM), in two kernels
// with the same arithmetic:
// (a) conv1d + SiLU and the q/k/v BlockLinears, one CTA per 256 channels and
//     four rows (a 4-channel block never straddles two CTAs); q and v to qkv,
//     the unscaled k to `kraw`;
// (b) one CTA per (head, row): the head's input and forget gate projections over
//     cat(q, k, v) with the CTA's threads splitting the 3*mi terms, then the
//     stabilized gates, the normalizer state and the denominator as in
//     k_mlstm_mid, and k / sqrt(hs) into qkv.
constexpr int kMidSplitRows = 64;  // steps up to this many rows take the two kernels
__global__ void __launch_bounds__(kRowThreads) k_mlstm_qkv_cols(const MlstmMidP p, float* kraw) {
  pdl_wait();
  constexpr int RM = 4;
  const int r0 = blockIdx.y * RM;
  const int nr = min(RM, live_rows(p.rc.n_dev, p.rc.rows) - r0);
  if (nr <= 0) return;
  const int mi = p.mi, tid = threadIdx.x;
  const int c = blockIdx.x * kRowThreads + tid;  // this thread's channel and q/k/v output
  __shared__ long long sslot[RM];
  __shared__ float4 xs4[RM][kRowThreads / 4];  // conv + SiLU of the CTA's channels, per row
  float* xs = reinterpret_cast<float*>(xs4);
  if (tid < nr) sslot[tid] = row_slot(p.rc, r0 + tid);
  __syncthreads();
  if (c < mi) {
    float s0[RM], s1[RM], s2[RM], xv[RM];
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      if (rr < nr) {
        const float* st = p.conv + sslot[rr] * p.cs;
        s0[rr] = st[c];
        s1[rr] = st[mi + c];
        s2[rr] = st[2 * mi + c];
        xv[rr] = p.proj[size_t(r0 + rr) * 2 * mi + c];
      }
    }
    const float w0 = p.cw[c], w1 = p.cw[mi + c], w2 = p.cw[2 * mi + c], w3 = p.cw[3 * mi + c], cb = p.cb[c];
#pragma unroll
    for (int rr = 0; rr < RM; ++rr) {
      if (rr < nr) {
        // CausalConv1d over [state, x] (model/modules.py:37-41)
        float acc = w0 * s0[rr];
        acc = fmaf(w1, s1[rr], acc);
        acc = fmaf(w2, s2[rr], acc);
        acc = fmaf(w3, xv[rr], acc);
        float* st = p.conv + sslot[rr] * p.cs;
        st[c] = s1[rr];
        st[mi + c] = s2[rr];
        st[2 * mi + c] = xv[rr];
        const float v = siluf_(acc + cb);
        xs[rr * kRowThreads + tid] = v;
        p.xca[size_t(r0 + rr) * mi + c] = v;
      }
    }
  }
  __syncthreads();
  if (c >= mi) return;
  // q/k from the conv branch, v from x_mlstm: 4x4 BlockLinear blocks (xlstm.py:209-211)
  const float4 wq = __ldg(reinterpret_cast<const float4*>(p.wq) + c);
  const float4 wk = __ldg(reinterpret_cast<const float4*>(p.wk) + c);
  const float4 wv = __ldg(reinterpret_cast<const float4*>(p.wv) + c);
#pragma unroll
  for (int rr = 0; rr < RM; ++rr) {
    if (rr >= nr) break;
    const int r = r0 + rr;
    const float4 xc = xs4[rr][tid >> 2];
    const float4 x0 = reinterpret_cast<const float4*>(p.proj + size_t(r) * 2 * mi)[c >> 2];
    p.qkv[size_t(r) * 3 * mi + c] = fmaf(xc.w, wq.w, fmaf(xc.z, wq.z, fmaf(xc.y, wq.y, xc.x * wq.x)));
    kraw[size_t(r) * mi + c] = fmaf(xc.w, wk.w, fmaf(xc.z, wk.z, fmaf(xc.y, wk.y, xc.x * wk.x)));
    p.qkv[size_t(r) * 3 * mi + 2 * mi + c] = fmaf(x0.w, wv.w, fmaf(x0.z, wv.z, fmaf(x0.y, wv.y, x0.x * wv.x)));
  }
}

__global__ void __launch_bounds__(kRowThreads) k_mlstm_cell_heads(const MlstmMidP p, const float* kraw) {
  prefetch_l2(p.gw + size_t(blockIdx.x) * 3 * p.mi, 3LL * p.mi);
  prefetch_l2(p.gw + size_t(p.nh + blockIdx.x) * 3 * p.mi, 3LL * p.mi);
  pdl_wait();
  const int h = blockIdx.x, r = blockIdx.y;
  if (!row_live(p.rc, r)) return;
  const int mi = p.mi, nh = p.nh, hs = p.hs, tid = threadIdx.x;
  __shared__ float red[2][kRowThreads / 32];
  const long long slot = row_slot(p.rc, r);
  const float* q = p.qkv + size_t(r) * 3 * mi;
  const float* kr = kraw + size_t(r) * mi;
  // igate / fgate of head h over cat(q, k, v) (xlstm.py:119-120), fp32
  const float4* wi = reinterpret_cast<const float4*>(p.gw + size_t(h) * 3 * mi);
  const float4* wf = reinterpret_cast<const float4*>(p.gw + size_t(nh + h) * 3 * mi);
  const int m4 = mi >> 2;
  float ai = 0.f, af = 0.f;
  constexpr int KU = 4;  // k steps whose loads are in flight together
  for (int k0 = tid; k0 < 3 * m4; k0 += KU * kRowThreads) {
    float4 xv[KU], av[KU], bv[KU];
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      const int k = k0 + u * kRowThreads;
      if (k < 3 * m4) {
        xv[u] = k < m4 ? reinterpret_cast<const float4*>(q)[k]
                       : (k < 2 * m4 ? reinterpret_cast<const float4*>(kr)[k - m4]
                                     : reinterpret_cast<const float4*>(q + 2 * mi)[k - 2 * m4]);
        av[u] = __ldg(wi + k);
        bv[u] = __ldg(wf + k);
      }
    }
#pragma unroll
    for (int u = 0; u < KU; ++u) {
      if (k0 + u * kRowThreads >= 3 * m4) break;
      const float4 x = xv[u], a = av[u], b = bv[u];
      ai = fmaf(x.w, a.w, fmaf(x.z, a.z, fmaf(x.y, a.y, fmaf(x.x, a.x, ai))));
      af = fmaf(x.w, b.w, fmaf(x.z, b.z, fmaf(x.y, b.y, fmaf(x.x, b.x, af))));
    }
  }
  ai = warp_sum(ai);
  af = warp_sum(af);
  if ((tid & 31) == 0) {
    red[0][tid >> 5] = ai;
    red[1][tid >> 5] = af;
  }
  __syncthreads();
  float ig = p.gb[h], fg = p.gb[nh + h];
  for (int w = 0; w < kRowThreads / 32; ++w) {
    ig += red[0][w];
    fg += red[1][w];
  }
  // MLSTMCell gates and normalizer (xlstm.py:92-103, 121-132)
  const float mo = p.m[slot * p.m_s + h];
  const float lf = logsigmoidf_(fg);
  const float mn = fmaxf(ig, mo + lf);
  const float i_g = expf(ig - mn), f_g = expf(lf + mo - mn);
  const float sq = sqrtf(float(hs));
  float* nst = p.n + slot * p.n_s;
  float qn = 0.f;
  for (int j0 = tid; j0 < hs; j0 += kEU * kRowThreads) {
    float kv[kEU], nv0[kEU], qv[kEU];
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int j = j0 + u * kRowThreads;
      if (j < hs) {
        const int e = h * hs + j;
        kv[u] = kr[e]; nv0[u] = nst[e]; qv[u] = q[e];
      }
    }
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int j = j0 + u * kRowThreads;
      if (j >= hs) break;
      const int e = h * hs + j;
      const float ks = kv[u] / sq;  // k / sqrt(head_size) (xlstm.py:99)
      const float nv = f_g * nv0[u] + i_g * ks;
      p.qkv[size_t(r) * 3 * mi + mi + e] = ks;
      nst[e] = nv;
      qn = fmaf(qv[u], nv, qn);
    }
  }
  qn = warp_sum(qn);
  __syncthreads();  // every thread has read red[] and m
  if ((tid & 31) == 0) red[0][tid >> 5] = qn;
  __syncthreads();
  if (tid == 0) {
    float v = 0.f;
    for (int w = 0; w < kRowThreads / 32; ++w) v += red[0][w];
    p.m[slot * p.m_s + h] = mn;
    p.g2[size_t(r) * 2 * nh + h] = i_g;
    p.g2[size_t(r) * 2 * nh + nh + h] = f_g;
    p.den[size_t(r) * nh + h] = fmaxf(fabsf(v), expf(-mn)) + 1e-6f;  // xlstm.py:130-132
  }
}

int mid_rows(int mi, int nh) {
  const size_t per = size_t(4 * mi + 2 * nh) * sizeof(float);
  B2E_CHECK(per <= kMidSmemMax, kErrInvalid, "mLSTM inner size too large for one CTA");
  return int(std::max<size_t>(1, std::min<size_t>(4, kMidSmemMax / per)));  // 4 = RM in k_mlstm_mid
}

struct MlstmPostP {
  RowCtx rc;
  const float* num; const float* den; const float* xca; const float* proj; int mi, nh;
  const float *gnw, *gnb, *skip; void* A; int at;
};
__global__ void __launch_bounds__(kRowThreads) k_mlstm_post(const MlstmPostP p) {
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  extern __shared__ float o[];
  __shared__ float gm[64], gr[64];
  const int hs = p.mi / p.nh;
  const float* num = p.num + size_t(r) * p.mi;
  for (int e = threadIdx.x; e < p.mi; e += blockDim.x) o[e] = num[e] / p.den[size_t(r) * p.nh + e / hs];  // xlstm.py:133
  __syncthreads();
  group_stats(o, p.nh, hs, 1e-5f, gm, gr);  // outnorm GroupNorm (xlstm.py:135)
  const float* xca = p.xca + size_t(r) * p.mi;
  const float* xg = p.proj + size_t(r) * 2 * p.mi + p.mi;
  for (int e = threadIdx.x; e < p.mi; e += blockDim.x) {
    const int g = e / hs;
    const float on = (o[e] - gm[g]) * gr[g] * p.gnw[e] + p.gnb[e];
    store_as(p.at, p.A, size_t(r) * p.mi + e, (on + p.skip[e] * xca[e]) * siluf_(xg[e]));  // xlstm.py:215-216
  }
}

// The same, one warp per (row, head): the head's hs = 32*T columns sit T to a
// lane, so GroupNorm's sums close with warp shuffles, with no shared memory,
// barrier or per-element division of indices. Heads of up to 512 columns.
constexpr int kPostWarps = 8;  // warps per CTA
template <int TM>  // columns per lane at most (hs <= 32 * TM)
__global__ void __launch_bounds__(256) k_mlstm_post_w(const MlstmPostP p) {
  prefetch_l1(p.gnw, p.mi);
  prefetch_l1(p.gnb, p.mi);
  prefetch_l1(p.skip, p.mi);
  pdl_wait();
  const int w = blockIdx.x * kPostWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int r = w / p.nh, g = w - r * p.nh;
  if (!row_live(p.rc, r)) return;
  const int mi = p.mi, hs = mi / p.nh, T = hs >> 5;
  const float* num = p.num + size_t(r) * mi;
  const float* xca = p.xca + size_t(r) * mi;
  const float* xg = p.proj + size_t(r) * 2 * mi + mi;
  {
    const float den = p.den[size_t(r) * p.nh + g];
    const int e0 = g * hs + lane;
    // every operand of the head's columns loaded before the first store
    float o[TM], gw[TM], gb[TM], sk[TM], xc[TM], xg2[TM];
#pragma unroll
    for (int t = 0; t < TM; ++t)
      if (t < T) {
        const int e = e0 + 32 * t;
        o[t] = num[e];
        gw[t] = p.gnw[e]; gb[t] = p.gnb[e]; sk[t] = p.skip[e]; xc[t] = xca[e]; xg2[t] = xg[e];
      }
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < TM; ++t)
      if (t < T) {
        o[t] = o[t] / den;  // xlstm.py:133
        s += o[t];
      }
    const float mu = warp_sum(s) / float(hs);
    float q = 0.f;
#pragma unroll
    for (int t = 0; t < TM; ++t)
      if (t < T) {
        const float d = o[t] - mu;
        q = fmaf(d, d, q);
      }
    const float rs = 1.0f / sqrtf(warp_sum(q) / float(hs) + 1e-5f);  // outnorm GroupNorm (xlstm.py:135)
#pragma unroll
    for (int t = 0; t < TM; ++t)
      if (t < T) {
        const int e = e0 + 32 * t;
        const float on = (o[t] - mu) * rs * gw[t] + gb[t];
        store_as(p.at, p.A, size_t(r) * mi + e, (on + sk[t] * xc[t]) * siluf_(xg2[t]));  // xlstm.py:215-216
      }
  }
}

struct XFinalP {
  RowCtx rc;
  const float* x2; int H; const float* w; const float* res; float* out;
};
__global__ void __launch_bounds__(kRowThreads) k_xlstm_final(const XFinalP p) {
  prefetch_l1(p.w, p.H);
  pdl_wait();
  const int r = blockIdx.x;
  if (!row_live(p.rc, r)) return;
  extern __shared__ float x[];
  __shared__ float gm[1], gr[1];
  for (int e = threadIdx.x; e < p.H; e += blockDim.x) x[e] = p.x2[size_t(r) * p.H + e];
  __syncthreads();
  group_stats(x, 1, p.H, 1e-5f, gm, gr);  // final LayerNorm (xlstm.py:365)
  for (int e0 = threadIdx.x; e0 < p.H; e0 += kEU * blockDim.x) {
    float wv[kEU], rv[kEU];
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e < p.H) {
        wv[u] = p.w[e];
        rv[u] = p.res ? p.res[size_t(r) * p.H + e] : 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < kEU; ++u) {
      const int e = e0 + u * blockDim.x;
      if (e >= p.H) break;
      const float y = (x[e] - gm[0]) * gr[0] * wv[u];
      p.out[size_t(r) * p.H + e] = p.res ? rv[u] + y : y;
    }
  }
}

class XLSTMLayer : public Layer {
 public:
  XLSTMLayer(const Dims& d, int lp) : d_(d), lp_(lp) {
    H_ = d.H; nbl_ = d.slstm_heads(); bs_ = d.slstm_bs();
    mi_ = d.mlstm_inner(); nh_ = d.mlstm_heads(); hs_ = d.mlstm_hs();
    B2E_CUDA(cudaFuncSetAttribute(k_mlstm_mid, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kMidSmemMax)));
    // the fused sLSTM kernel: one thread per hidden unit, 16-byte activation
    // vectors inside a block, kSlRows rows of three activation planes in smem
    fused_ = H_ % 32 == 0 && H_ >= sl_rows() && H_ <= 512 && bs_ % 4 == 0 && nbl_ <= kSlMaxGroups &&
             fused_smem() <= kSlSmemMax;
    if (fused_) {
      B2E_CUDA(cudaFuncSetAttribute(k_slstm_fused<kSlRows, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(fused_smem())));
      B2E_CUDA(cudaFuncSetAttribute(k_slstm_fused<kSlRows, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(fused_smem())));
      B2E_CUDA(cudaFuncSetAttribute(k_slstm_fused<kSlRowsNarrow, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(fused_smem())));
    }
  }
  int sl_rows() const { return H_ <= 128 ? kSlRowsNarrow : kSlRows; }
  size_t fused_smem() const { return size_t(3) * sl_rows() * H_ * sizeof(float); }
  void declare_state(StateArena& a) override {
    // (xlstm.py:331-336, 276-282, 232-236, 150-156) in init_state order
    l_sconv_ = a.add_conv(H_, 3);
    l_sh_ = a.add(H_);
    l_sc_ = a.add(H_);
    l_sn_ = a.add(H_);
    l_sm_ = a.add(H_, kLeafF32, -INFINITY);
    l_mconv_ = a.add_conv(mi_, 3);
    l_C_ = a.add(nh_ * hs_ * hs_);
    l_n_ = a.add(nh_ * hs_);
    l_m_ = a.add(nh_);
  }
  void load(WeightSource& s, WeightPack& w, const std::string& p) override {
    const size_t H = H_, BB = size_t(nbl_) * bs_ * bs_;
    o_slnw_ = w.add(s.get(p + "slstm.norm.weight", H), H, kF32);
    o_scw_ = w.add_conv(s.get(p + "slstm.conv1d.conv.weight", H * 4), H_, 4);
    o_scb_ = w.add(s.get(p + "slstm.conv1d.conv.bias", H), H, kF32);
    // Wcat[g][j] = [W_input_g[j] | W_state_g[j]]  (bs x 2bs), gates in order i, f, z, o
    const char* gates = "ifzo";
    std::vector<const float*> win(4), wst(4), bst(4);
    for (int g = 0; g < 4; ++g) {
      const std::string gn(1, gates[g]);
      win[g] = s.get(p + "slstm." + gn + "gate_input.weight", BB);
      wst[g] = s.get(p + "slstm." + gn + "gate_state.weight", BB);
      bst[g] = s.get(p + "slstm." + gn + "gate_state.bias", H);
    }
    const int nbl = nbl_, bs = bs_;
    o_swcat_ = w.reserve(size_t(4) * nbl * bs * 2 * bs * 4, [=](uint8_t* dst) {
      float* o = reinterpret_cast<float*>(dst);
      for (int g = 0; g < 4; ++g)
        for (int j = 0; j < nbl; ++j)
          for (int e = 0; e < bs; ++e) {
            float* row = o + ((size_t(g) * nbl + j) * bs + e) * 2 * bs;
            const float* a = win[g] + (size_t(j) * bs + e) * bs;
            const float* b = wst[g] + (size_t(j) * bs + e) * bs;
            std::copy(a, a + bs, row);
            std::copy(b, b + bs, row + bs);
          }
    });
    if (fused_) {
      // Wt[k][g][u]: k < bs the input half, k >= bs the state half, u = j*bs + e
      o_swt_ = w.reserve(size_t(4) * 2 * bs * H * 4, [=](uint8_t* dst) {
        float* o = reinterpret_cast<float*>(dst);
        const size_t Hs = H;
        for (int k = 0; k < 2 * bs; ++k)
          for (int g = 0; g < 4; ++g)
            for (size_t u = 0; u < Hs; ++u)
              o[(size_t(k) * 4 + g) * Hs + u] = k < bs ? win[g][u * bs + k] : wst[g][u * bs + (k - bs)];
      });
    }
    o_sbias_ = w.add_rows({{bst[0], H}, {bst[1], H}, {bst[2], H}, {bst[3], H}}, kF32);
    o_sgnw_ = w.add(s.get(p + "slstm.group_norm.weight", H), H, kF32);
    o_sgnb_ = w.add(s.get(p + "slstm.group_norm.bias", H), H, kF32);
    const size_t mi = mi_, QB = size_t(mi_ / 4) * 16;
    o_skip_ = w.add(s.get(p + "mlstm.learnable_skip", mi), mi, kF32);
    o_mlnw_ = w.add(s.get(p + "mlstm.norm.weight", H), H, kF32);
    o_mw1_ = w.add_rows({{s.get(p + "mlstm.x_proj.weight", mi * H), mi * H},
                         {s.get(p + "mlstm.gate_proj.weight", mi * H), mi * H}}, lp_);
    o_wq_ = w.add(s.get(p + "mlstm.q_proj.weight", QB), QB, kF32);
    o_wk_ = w.add(s.get(p + "mlstm.k_proj.weight", QB), QB, kF32);
    o_wv_ = w.add(s.get(p + "mlstm.v_proj.weight", QB), QB, kF32);
    o_mcw_ = w.add_conv(s.get(p + "mlstm.conv1d.conv.weight", mi * 4), mi_, 4);
    o_mcb_ = w.add(s.get(p + "mlstm.conv1d.conv.bias", mi), mi, kF32);
    const std::string cp = p + "mlstm.mlstm_cell.";
    const size_t GW = size_t(nh_) * 3 * mi;
    o_gw_ = w.add_rows({{s.get(cp + "igate_proj.weight", GW), GW}, {s.get(cp + "fgate_proj.weight", GW), GW}}, kF32);
    o_gb_ = w.add_rows({{s.get(cp + "igate_proj.bias", nh_), size_t(nh_)},
                        {s.get(cp + "fgate_proj.bias", nh_), size_t(nh_)}}, kF32);
    o_ongw_ = w.add(s.get(cp + "outnorm.weight", mi), mi, kF32);
    o_ongb_ = w.add(s.get(cp + "outnorm.bias", mi), mi, kF32);
    o_down_ = w.add(s.get(p + "mlstm.proj_down.weight", H * mi), H * mi, lp_);
    o_fnw_ = w.add(s.get(p + "final_norm.weight", H), H, kF32);
  }
  void resolve(const WeightPack& w, const StateArena& a) override {
    slnw_ = w.ptr<float>(o_slnw_); scw_ = w.ptr<float>(o_scw_); scb_ = w.ptr<float>(o_scb_);
    swcat_ = w.ptr<float>(o_swcat_); sbias_ = w.ptr<float>(o_sbias_);
    swt_ = fused_ ? w.ptr<float>(o_swt_) : nullptr;
    sgnw_ = w.ptr<float>(o_sgnw_); sgnb_ = w.ptr<float>(o_sgnb_);
    skip_ = w.ptr<float>(o_skip_); mlnw_ = w.ptr<float>(o_mlnw_); mw1_ = w.ptr(o_mw1_);
    wq_ = w.ptr<float>(o_wq_); wk_ = w.ptr<float>(o_wk_); wv_ = w.ptr<float>(o_wv_);
    mcw_ = w.ptr<float>(o_mcw_); mcb_ = w.ptr<float>(o_mcb_); gw_ = w.ptr<float>(o_gw_); gb_ = w.ptr<float>(o_gb_);
    ongw_ = w.ptr<float>(o_ongw_); ongb_ = w.ptr<float>(o_ongb_); down_ = w.ptr(o_down_); fnw_ = w.ptr<float>(o_fnw_);
    sconv_ = a.f32(l_sconv_); sh_ = a.f32(l_sh_); sc_ = a.f32(l_sc_); sn_ = a.f32(l_sn_); sm_ = a.f32(l_sm_);
    mconv_ = a.f32(l_mconv_); C_ = a.f32(l_C_); n_ = a.f32(l_n_); m_ = a.f32(l_m_);
    ssconv_ = a.stride(l_sconv_); ssh_ = a.stride(l_sh_); ssc_ = a.stride(l_sc_); ssn_ = a.stride(l_sn_);
    ssm_ = a.stride(l_sm_); smconv_ = a.stride(l_mconv_); sC_ = a.stride(l_C_); sn2_ = a.stride(l_n_);
    sm2_ = a.stride(l_m_);
  }
  struct Buf { float *axc, *axn, *G, *x1, *xn2, *proj, *xca, *qkv, *g2, *den, *num, *A, *x2; };
  Buf carve(uint8_t* base, int rows) const {
    Carver c{base};
    Buf b;
    const size_t R = rows;
    b.axc = c.take<float>(R * 2 * H_);
    b.axn = c.take<float>(R * 2 * H_);
    b.G = c.take<float>(R * 4 * H_);
    b.x1 = c.take<float>(R * H_);
    b.xn2 = c.take<float>(R * H_);
    b.proj = c.take<float>(R * 2 * mi_);
    b.xca = c.take<float>(R * mi_);
    b.qkv = c.take<float>(R * 3 * mi_);
    b.g2 = c.take<float>(R * 2 * nh_);
    b.den = c.take<float>(R * nh_);
    b.num = c.take<float>(R * mi_);
    b.A = c.take<float>(R * mi_);
    b.x2 = c.take<float>(R * H_);
    scratch_ = c.off;
    return b;
  }
  size_t scratch_bytes(int rows) const override {
    carve(nullptr, rows);
    return scratch_;
  }
  void forward(const StepCtx& c, const float* in, const void* in_lp, float* out, const float* residual,
               uint8_t* scratch, const RowEpi* post) override {
    const Buf b = carve(scratch, c.rows);
    const RowCtx rc{c.n_dev, c.rows, c.slots};
    // ---- sLSTM block (xlstm.py:304-318)
    if (fused_) {
      SlstmFusedP fp{rc, in, H_, nbl_, bs_, slnw_, sconv_, ssconv_, scw_, scb_, sh_, sc_, sn_, sm_, ssh_, ssc_, ssn_, ssm_,
                     swt_, sbias_, sgnw_, sgnb_, mlnw_, b.x1, b.xn2, lp_};
      if (H_ == 256)
        launch_k(c.ln, k_slstm_fused<kSlRows, 256>, dim3(ceil_div(c.rows, kSlRows)), dim3(H_), fused_smem(), c.s, fp);
      else if (sl_rows() == kSlRowsNarrow)
        launch_k(c.ln, k_slstm_fused<kSlRowsNarrow, 0>, dim3(ceil_div(c.rows, kSlRowsNarrow)), dim3(H_), fused_smem(),
                 c.s, fp);
      else
        launch_k(c.ln, k_slstm_fused<kSlRows, 0>, dim3(ceil_div(c.rows, kSlRows)), dim3(H_), fused_smem(), c.s, fp);
    } else {
      SlstmPreP sp{rc, in, H_, nbl_, bs_, slnw_, sconv_, ssconv_, scw_, scb_, sh_, ssh_, b.axc, b.axn};
      launch_k(c.ln, k_slstm_pre, dim3(c.rows), dim3(kRowThreads), H_ * sizeof(float), c.s, sp);
      // i, f from the conv branch, z, o from the normed input, each + BlockLinear(h) + bias (xlstm.py:312-315)
      for (int g0 = 0; g0 < 4 * nbl_; g0 += kMaxGroups) {
        GemmParams gp;
        gp.groups = std::min(kMaxGroups, 4 * nbl_ - g0);
        for (int q = 0; q < gp.groups; ++q) {
          const int gi = g0 + q, g = gi / nbl_, j = gi % nbl_;
          GemmGroup& gg = gp.g[q];
          gg.A = (g < 2 ? b.axc : b.axn) + size_t(j) * 2 * bs_;
          gg.W = swcat_ + size_t(gi) * bs_ * 2 * bs_;
          gg.bias = sbias_ + size_t(g) * H_ + j * bs_;
          gg.C = b.G + size_t(g) * H_ + j * bs_;
        }
        gp.M_max = c.rows; gp.M_dev = c.n_dev; gp.N = bs_; gp.K = 2 * bs_;
        gp.lda = 2 * H_; gp.ldw = 2 * bs_; gp.ldc = 4 * H_;
        gp.ln = c.ln;
        gemm(gp, c.s);
      }
      SlstmPostP so{rc, b.G, in, H_, nbl_, sh_, sc_, sn_, sm_, ssh_, ssc_, ssn_, ssm_, sgnw_, sgnb_, mlnw_, b.x1, b.xn2, lp_};
      launch_k(c.ln, k_slstm_post, dim3(c.rows), dim3(kRowThreads), 2 * H_ * sizeof(float), c.s, so);
    }
    // ---- mLSTM block (xlstm.py:198-219)
    linear(c, b.xn2, lp_, H_, mw1_, lp_, nullptr, 2 * mi_, H_, b.proj, 2 * mi_);  // x_proj, gate_proj
    const int rpc = mid_rows(mi_, nh_);
    MlstmMidP mp{rc, b.proj, mi_, nh_, hs_, mconv_, smconv_, mcw_, mcb_, wq_, wk_, wv_, gw_, gb_,
                 n_, sn2_, m_, sm2_, b.xca, b.qkv, b.g2, b.den, rpc};
    if (c.rows <= kMidSplitRows) {
      // b.num (written by the state step below) holds the unscaled k meanwhile
      launch_k(c.ln, k_mlstm_qkv_cols, dim3(ceil_div(mi_, kRowThreads), ceil_div(c.rows, 4)), dim3(kRowThreads), 0,
               c.s, mp, b.num);
      launch_k(c.ln, k_mlstm_cell_heads, dim3(nh_, c.rows), dim3(kRowThreads), 0, c.s, mp,
               static_cast<const float*>(b.num));
    } else {
      launch_k(c.ln, k_mlstm_mid, dim3(ceil_div(c.rows, rpc)), dim3(kRowThreads),
               size_t(rpc) * (4 * mi_ + 2 * nh_) * sizeof(float), c.s, mp);
    }
    OuterRowsParams op;
    op.at = {C_, sC_, c.slots, nullptr, c.rows, c.n_dev};
    op.nh = nh_; op.sh = hs_; op.sk = hs_;
    op.f = b.g2 + nh_; op.f_rs = 2 * nh_; op.f_hs = 1;
    op.i = b.g2; op.i_rs = 2 * nh_; op.i_hs = 1;
    op.kv = b.qkv + mi_; op.k_rs = 3 * mi_;
    op.v = b.qkv + 2 * mi_; op.v_rs = 3 * mi_;
    op.q = b.qkv; op.q_rs = 3 * mi_;
    op.out = b.num; op.o_rs = mi_;
    op.err = c.err;
    outer_rows(op, c.rows, c.s, c.ln_bulk);
    MlstmPostP pp{rc, b.num, b.den, b.xca, b.proj, mi_, nh_, ongw_, ongb_, skip_, b.A, lp_};
    if (hs_ % 32 == 0 && hs_ <= 512) {
      const dim3 pg(ceil_div(c.rows * nh_, kPostWarps));
      const int T = hs_ / 32;
      if (T <= 2)
        launch_k(c.ln, k_mlstm_post_w<2>, pg, dim3(256), 0, c.s, pp);
      else if (T <= 4)
        launch_k(c.ln, k_mlstm_post_w<4>, pg, dim3(256), 0, c.s, pp);
      else if (T <= 8)
        launch_k(c.ln, k_mlstm_post_w<8>, pg, dim3(256), 0, c.s, pp);
      else
        launch_k(c.ln, k_mlstm_post_w<16>, pg, dim3(256), 0, c.s, pp);
    } else {
      launch_k(c.ln, k_mlstm_post, dim3(c.rows), dim3(kRowThreads), mi_ * sizeof(float), c.s, pp);
    }
    if (post) {
      // proj_down + skip, final LayerNorm, Block residual and the Block's norm2,
      // all in the GEMM epilogue (xlstm.py:217-219, 365; inference_model.py:65-67)
      RowEpi re = *post;
      re.ln_w = fnw_;
      re.ln_eps = 1e-5f;
      re.R2 = residual;
      re.ldr2 = H_;
      linear(c, b.A, lp_, mi_, down_, lp_, nullptr, H_, mi_, out, H_, kActNone, b.x1, H_, nullptr, 0, &re);
    } else {
      linear(c, b.A, lp_, mi_, down_, lp_, nullptr, H_, mi_, b.x2, H_, kActNone, b.x1, H_);  // proj_down + skip
      XFinalP fp{rc, b.x2, H_, fnw_, residual, out};
      launch_k(c.ln, k_xlstm_final, dim3(c.rows), dim3(kRowThreads), H_ * sizeof(float), c.s, fp);
    }
    B2E_CUDA(cudaGetLastError());
  }

  void latency_desc(LatLayer& L) const override {
    const void* w[] = {slnw_, scw_, scb_, swcat_, sbias_, sgnw_, sgnb_, skip_, mlnw_, mw1_, wq_,
                       wk_, wv_, mcw_, mcb_, gw_, gb_, ongw_, ongb_, down_, fnw_};
    for (size_t k = 0; k < sizeof(w) / sizeof(w[0]); ++k) L.w[k] = w[k];
    float* st[] = {sconv_, sh_, sc_, sn_, sm_, mconv_, C_, n_, m_};
    const long long ss[] = {ssconv_, ssh_, ssc_, ssn_, ssm_, smconv_, sC_, sn2_, sm2_};
    for (int k = 0; k < 9; ++k) { L.st[k] = st[k]; L.ss[k] = ss[k]; }
  }

 private:
  Dims d_;
  int lp_, H_, nbl_, bs_, mi_, nh_, hs_;
  mutable size_t scratch_ = 0;
  int l_sconv_, l_sh_, l_sc_, l_sn_, l_sm_, l_mconv_, l_C_, l_n_, l_m_;
  bool fused_ = false;
  size_t o_swt_ = 0;
  const float* swt_ = nullptr;
  size_t o_slnw_, o_scw_, o_scb_, o_swcat_, o_sbias_, o_sgnw_, o_sgnb_, o_skip_, o_mlnw_, o_mw1_, o_wq_, o_wk_,
      o_wv_, o_mcw_, o_mcb_, o_gw_, o_gb_, o_ongw_, o_ongb_, o_down_, o_fnw_;
  const float *slnw_, *scw_, *scb_, *swcat_, *sbias_, *sgnw_, *sgnb_, *skip_, *mlnw_, *wq_, *wk_, *wv_, *mcw_,
      *mcb_, *gw_, *gb_, *ongw_, *ongb_, *fnw_;
  const void *mw1_ = nullptr, *down_ = nullptr;
  float *sconv_, *sh_, *sc_, *sn_, *sm_, *mconv_, *C_, *n_, *m_;
  long long ssconv_, ssh_, ssc_, ssn_, ssm_, smconv_, sC_, sn2_, sm2_;
};

}  // namespace

// ------------------------------------------------------------ public glue

std::unique_ptr<Layer> Layer::make(int kind, const Dims& d, int lp) {
  switch (kind) {
    case kXLSTM: return std::make_unique<XLSTMLayer>(d, lp);
    case kMamba2: return std::make_unique<Mamba2Layer>(d, lp);
    case kRetNet: return std::make_unique<RetNetLayer>(d, lp);
    case kHawk: return std::make_unique<HawkLayer>(d, lp);
  }
  throw Error(kErrInvalid, "unknown layer kind " + std::to_string(kind));
}

void rmsnorm_rows(const StepCtx& c, const float* x, const float* w, float eps, int H, float* out, void* out_lp) {
  RmsP p{{c.n_dev, c.rows, c.slots}, x, w, out, H, eps, out_lp, c.lp};
  launch_k(c.ln, k_rmsnorm, dim3(ceil_div(c.rows, kRowsPerCta)), dim3(256), 0, c.s, p);
  B2E_CUDA(cudaGetLastError());
}

void output_proj_rows(const StepCtx& c, const float* x, const float* w, const float* b, int H, float* preds, int ld,
                      int col) {
  OutP p{{c.n_dev, c.rows, c.slots}, x, w, b, H, preds, ld, col};
  launch_k(c.ln, k_output_proj, dim3(ceil_div(c.rows, kRowsPerCta)), dim3(256), 0, c.s, p);
  B2E_CUDA(cudaGetLastError());
}

bool fused_rows(const StepCtx& c, int H) { return c.lp != kF32 && c.rows > 16 && H <= 256 && H % 16 == 0; }

void linear(const StepCtx& c, const void* A, int at, int lda, const void* W, int wt, const void* bias, int N, int K,
            float* C, int ldc, int act, const float* R, int ldr, void* C_lp, int ldc_lp, const RowEpi* row) {
  GemmParams p;
  p.groups = 1;
  p.g[0].A = A;
  p.g[0].W = W;
  p.g[0].bias = bias;
  p.g[0].C = C;
  p.g[0].R = R;
  p.g[0].C_lp = C_lp;
  p.ldc_lp = ldc_lp;
  p.err = c.err;
  p.M_max = c.rows;
  p.M_dev = c.n_dev;
  p.N = N;
  p.K = K;
  p.lda = lda;
  p.ldw = K;
  p.ldc = ldc;
  p.ldr = ldr;
  p.a_type = at;
  p.w_type = wt;
  p.bias_type = wt;  // CastLinear stores its bias in the weight's type (example_model.py:85-88)
  p.round_out = wt != kF32;
  p.act = act;
  p.ln = c.ln;
  if (row) {
    p.row = *row;
    B2E_CHECK(gemm_tc_row_eligible(p), kErrInternal, "fused row epilogue requested for an ineligible projection");
  }
  gemm(p, c.s);
}

void set_rows(int* n_dev, int n, cudaStream_t s) {
  k_set_rows<<<1, 1, 0, s>>>(n_dev, n);
  B2E_CUDA(cudaGetLastError());
}

}  // namespace b2e
