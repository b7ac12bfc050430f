// State-streaming recurrent steps (see cells.cuh).
//
// Memory plan: one CTA owns one (row, head, tile) of the state. Every thread
// moves 16-byte vectors with evict-first loads/stores and keeps four of them in
// flight before it computes, so a 148-SM part has ~100 KB of loads outstanding
// per SM - enough to cover HBM latency at full bandwidth. The small per-row
// operands (q, i*k, v or dt*b, c, x) are staged once in shared memory.
#include "cells.cuh"
#include "stream.cuh"

#include <algorithm>

namespace b2e {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxSh = 512;   // largest contracted/carried head axis kept in smem
constexpr int kKT = 128;      // k-columns per CTA in outer_rows

__device__ __forceinline__ int row_slot(const RowAddr& a, int row) { return a.slots ? a.slots[row] : row; }

// outer_rows: one CTA = (row, group of HG heads, tile of kw <= 128 carried
// columns). Work item = one 16-byte vector (h, 4 columns) of one head; thread t
// owns column vector c4 = t % L and state rows h = hr, hr + RH, ... of every head
// in the group, so a warp reads contiguous 512-byte runs. Each thread keeps two
// batches of U vectors in flight; the first batch is issued before the per-row
// operands are staged in shared memory, so the two latencies overlap.
constexpr int U = 4;

__global__ void __launch_bounds__(kThreads) outer_rows_kernel(const __grid_constant__ OuterRowsParams p, int HG) {
  pdl_wait();
  const int row = blockIdx.z;
  if (row >= live_rows(p.at.n_dev, p.at.n_host)) return;
  const int h0 = blockIdx.y * HG;
  const int hg = min(HG, p.nh - h0);
  const int k0 = blockIdx.x * kKT;
  const int kw = min(kKT, p.sk - k0);
  const int tid = threadIdx.x;
  const int L = kw >> 2, RH = kThreads / L;
  const int c4 = tid % L, hr = tid / L;
  const bool worker = hr < RH;
  const int pairs = hg * p.sh;  // (head, state row) pairs of this CTA

  if (p.at.mask && !p.at.mask[row]) {  // idle: state untouched, output zero
    for (int i = tid; i < hg * kw; i += kThreads)
      p.out[size_t(row) * p.o_rs + size_t(h0 + i / kw) * p.sk + k0 + i % kw] = 0.0f;
    return;
  }
  float* S = p.at.state + size_t(row_slot(p.at, row)) * p.at.row_stride + size_t(h0) * p.sh * p.sk + k0 + c4 * 4;
  auto addr = [&](int pi) { return S + (size_t(pi / p.sh) * p.sh + pi % p.sh) * p.sk; };  // pi = hh*sh + h

  float4 cur[U], nxt[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int pi = hr + u * RH;
    if (worker && pi < pairs) cur[u] = ld_stream(reinterpret_cast<const float4*>(addr(pi)));
  }

  extern __shared__ __align__(16) float sm[];
  const int qn = (HG * p.sh + 3) & ~3;   // every sub-array starts 16-byte aligned
  float* qs = sm;                        // [hg][sh]
  float* iks = qs + qn;                  // [hg][sh]  i * k
  float* vs = iks + qn;                  // [hg][kKT]
  float* fs = vs + HG * kKT;             // [hg]
  float* part = fs + ((HG + 3) & ~3);    // [hg][RH][kw], zeroed: a thread row may skip a head
  for (int i = tid; i < hg * RH * kw; i += kThreads) part[i] = 0.0f;
  for (int i = tid; i < hg * p.sh; i += kThreads) {
    const int hh = i / p.sh, h = i - hh * p.sh, n = h0 + hh;
    const float ii = p.i ? p.i[size_t(row) * p.i_rs + size_t(n) * p.i_hs] : 1.0f;
    qs[i] = p.q[size_t(row) * p.q_rs + size_t(n) * p.sh + h];
    iks[i] = ii * p.kv[size_t(row) * p.k_rs + size_t(n) * p.sh + h];
  }
  for (int i = tid; i < hg * kw; i += kThreads) {
    const int hh = i / kw, k = i - hh * kw;
    vs[hh * kKT + k] = p.v[size_t(row) * p.v_rs + size_t(h0 + hh) * p.sk + k0 + k];
  }
  for (int hh = tid; hh < hg; hh += kThreads) fs[hh] = p.f[size_t(row) * p.f_rs + size_t(h0 + hh) * p.f_hs];
  __syncthreads();

  if (worker) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int cur_hh = -1;
    for (int base = 0; base < pairs; base += U * RH) {
      const int nbase = base + U * RH;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int pi = nbase + hr + u * RH;
        if (pi < pairs) nxt[u] = ld_stream(reinterpret_cast<const float4*>(addr(pi)));
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int pi = base + hr + u * RH;
        if (pi < pairs) {
          const int hh = pi / p.sh;
          if (hh != cur_hh) {
            if (cur_hh >= 0) *reinterpret_cast<float4*>(&part[(cur_hh * RH + hr) * kw + c4 * 4]) = acc;
            acc = make_float4(0.f, 0.f, 0.f, 0.f);
            cur_hh = hh;
          }
          const float f = fs[hh], ik = iks[pi], qh = qs[pi];
          const float4 v4 = *reinterpret_cast<const float4*>(&vs[hh * kKT + c4 * 4]);
          float4 nv;
          nv.x = fmaf(f, cur[u].x, ik * v4.x);
          nv.y = fmaf(f, cur[u].y, ik * v4.y);
          nv.z = fmaf(f, cur[u].z, ik * v4.z);
          nv.w = fmaf(f, cur[u].w, ik * v4.w);
          st_stream(reinterpret_cast<float4*>(addr(pi)), nv);
          acc.x = fmaf(qh, nv.x, acc.x);
          acc.y = fmaf(qh, nv.y, acc.y);
          acc.z = fmaf(qh, nv.z, acc.z);
          acc.w = fmaf(qh, nv.w, acc.w);
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) cur[u] = nxt[u];
    }
    if (cur_hh >= 0) *reinterpret_cast<float4*>(&part[(cur_hh * RH + hr) * kw + c4 * 4]) = acc;
  }
  __syncthreads();
  for (int i = tid; i < hg * kw; i += kThreads) {
    const int hh = i / kw, k = i - hh * kw;
    // thread (hr, c4) summed the rows h of head hh it owns; slots it did not own are zero
    float sum = 0.f;
    for (int r = 0; r < RH; ++r) sum += part[(hh * RH + r) * kw + k];
    p.out[size_t(row) * p.o_rs + size_t(h0 + hh) * p.sk + k0 + k] = sum;
  }
}

// ssm_cols: one CTA = (row, group of HG heads, tile of pw state rows p). Work
// item = one 16-byte vector (p, 4 state columns c); the contraction over c closes
// inside the CTA. Same two-batch prefetch as outer_rows.
__global__ void __launch_bounds__(kThreads) ssm_cols_kernel(const __grid_constant__ SsmColsParams p, int PT, int HG) {
  pdl_wait();
  const int row = blockIdx.z;
  if (row >= live_rows(p.at.n_dev, p.at.n_host)) return;
  const int h0 = blockIdx.y * HG;
  const int hg = min(HG, p.nh - h0);
  const int p0 = blockIdx.x * PT;
  const int pw = min(PT, p.sh - p0);
  const int tid = threadIdx.x;
  const int LC = p.sc >> 2;
  const int per_head = pw * LC;
  const int items = hg * per_head;

  if (p.at.mask && !p.at.mask[row]) {
    for (int i = tid; i < hg * pw; i += kThreads)
      p.out[size_t(row) * p.o_rs + size_t(h0 + i / pw) * p.sh + p0 + i % pw] = 0.0f;
    return;
  }
  float* H = p.at.state + size_t(row_slot(p.at, row)) * p.at.row_stride;
  // item it -> head hh = it / per_head, then (p, c4) inside that head's [p0, p0+pw) rows
  auto addr = [&](int it) {
    const int hh = it / per_head, r = it - hh * per_head;
    return H + ((size_t(h0 + hh) * p.sh + p0) * p.sc) + size_t(r) * 4;
  };

  float4 cur[U], nxt[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int it = tid + u * kThreads;
    if (it < items) cur[u] = ld_stream(reinterpret_cast<const float4*>(addr(it)));
  }

  extern __shared__ __align__(16) float sm[];
  float* bs = sm;                       // b[c]
  float* cs = bs + p.sc;                // c[c]
  float* dts = cs + p.sc;               // dt per head
  float* dcs = dts + ((HG + 3) & ~3);   // decay per head
  float* xs = dcs + ((HG + 3) & ~3);    // [hg][pw] x
  float* part = xs + ((HG * PT + 3) & ~3);  // [items]
  for (int c = tid; c < p.sc; c += kThreads) {
    bs[c] = p.b[size_t(row) * p.b_rs + c];
    cs[c] = p.c[size_t(row) * p.c_rs + c];
  }
  for (int hh = tid; hh < hg; hh += kThreads) {
    dts[hh] = p.dt[size_t(row) * p.dt_rs + h0 + hh];
    dcs[hh] = p.decay[size_t(row) * p.dc_rs + h0 + hh];
  }
  for (int i = tid; i < hg * pw; i += kThreads) {
    const int hh = i / pw, pp = i - hh * pw;
    xs[i] = p.x[size_t(row) * p.x_rs + size_t(h0 + hh) * p.sh + p0 + pp];
  }
  __syncthreads();

  for (int base = 0; base < items; base += U * kThreads) {
    const int nbase = base + U * kThreads;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = nbase + tid + u * kThreads;
      if (it < items) nxt[u] = ld_stream(reinterpret_cast<const float4*>(addr(it)));
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int it = base + tid + u * kThreads;
      if (it < items) {
        const int hh = it / per_head, r = it - hh * per_head;
        const int pi = r / LC, c4 = r - pi * LC;
        const float dt = dts[hh], dc = dcs[hh], xp = xs[hh * pw + pi];
        const float4 b4 = *reinterpret_cast<const float4*>(&bs[c4 * 4]);
        const float4 c4v = *reinterpret_cast<const float4*>(&cs[c4 * 4]);
        float4 nv;  // decay*h + (dt*b)*x  (model/kernels.py:163-171)
        nv.x = fmaf(dc, cur[u].x, (dt * b4.x) * xp);
        nv.y = fmaf(dc, cur[u].y, (dt * b4.y) * xp);
        nv.z = fmaf(dc, cur[u].z, (dt * b4.z) * xp);
        nv.w = fmaf(dc, cur[u].w, (dt * b4.w) * xp);
        st_stream(reinterpret_cast<float4*>(addr(it)), nv);
        part[it] = fmaf(c4v.w, nv.w, fmaf(c4v.z, nv.z, fmaf(c4v.y, nv.y, c4v.x * nv.x)));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) cur[u] = nxt[u];
  }
  __syncthreads();
  for (int i = tid; i < hg * pw; i += kThreads) {
    const int hh = i / pw, pp = i - hh * pw;
    const float* pr = part + hh * per_head + pp * LC;
    float sum = 0.f;
    for (int c4 = 0; c4 < LC; ++c4) sum += pr[c4];
    p.out[size_t(row) * p.o_rs + size_t(h0 + hh) * p.sh + p0 + pp] = sum;
  }
}

// ---- fast paths: a thread owns one 16-byte column vector for the CTA's life and
// walks its state rows by pointer increments (no integer division per item).

// Mamba2, sc/4 = LC in {8, 16, 32}: LC lanes of one warp cover one state row p,
// so y[p] = sum_c c[c]*H_new[p,c] closes with log2(LC) shuffles.
template <int LC>
__global__ void __launch_bounds__(kThreads, 4) ssm_cols_fast(const __grid_constant__ SsmColsParams p, int PT, int HG) {
  pdl_wait();
  const int row = blockIdx.z;
  if (row >= live_rows(p.at.n_dev, p.at.n_host)) return;
  constexpr int RP = kThreads / LC;  // state rows in flight per pass
  const int h0 = blockIdx.y * HG;
  const int hg = min(HG, p.nh - h0);
  const int p0 = blockIdx.x * PT;
  const int pw = min(PT, p.sh - p0);
  const int tid = threadIdx.x;
  const int c4 = tid % LC, pr = tid / LC;
  if (p.at.mask && !p.at.mask[row]) {
    for (int i = tid; i < hg * pw; i += kThreads)
      p.out[size_t(row) * p.o_rs + size_t(h0 + i / pw) * p.sh + p0 + i % pw] = 0.0f;
    return;
  }
  const int per = pr < pw ? (pw - pr + RP - 1) / RP : 0;  // state rows per head for this thread
  const size_t sc = size_t(LC) * 4;
  float* H = p.at.state + size_t(row_slot(p.at, row)) * p.at.row_stride + (size_t(h0) * p.sh + p0 + pr) * sc + c4 * 4;

  // first batch before the operands are staged
  float4 cur[U];
  int hh_l = 0, k_l = 0;  // next item to load: head hh_l, k_l-th of this thread's rows
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (hh_l < hg && per > 0) {
      cur[u] = ld_stream(reinterpret_cast<const float4*>(H + (size_t(hh_l) * p.sh + size_t(k_l) * RP) * sc));
      if (++k_l == per) { k_l = 0; ++hh_l; }
    }
  }
  extern __shared__ __align__(16) float sm[];
  float* xs = sm;                         // [hg][pw]
  float* dts = xs + ((HG * PT + 3) & ~3); // [hg]
  float* dcs = dts + ((HG + 3) & ~3);     // [hg]
  for (int i = tid; i < hg * pw; i += kThreads) {
    const int hh = i / pw, pp = i - hh * pw;
    xs[i] = p.x[size_t(row) * p.x_rs + size_t(h0 + hh) * p.sh + p0 + pp];
  }
  for (int hh = tid; hh < hg; hh += kThreads) {
    dts[hh] = p.dt[size_t(row) * p.dt_rs + h0 + hh];
    dcs[hh] = p.decay[size_t(row) * p.dc_rs + h0 + hh];
  }
  const float4 b4 = *reinterpret_cast<const float4*>(p.b + size_t(row) * p.b_rs + c4 * 4);
  const float4 cv = *reinterpret_cast<const float4*>(p.c + size_t(row) * p.c_rs + c4 * 4);
  __syncthreads();

  int hh_c = 0, k_c = 0;  // next item to compute
  const int total = hg * per;
  // every lane runs the same number of rounds (the shuffles below need the whole warp)
  const int rounds = hg * ((pw + RP - 1) / RP);
  for (int done = 0; done < rounds; done += U) {
    float4 nxt[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (hh_l < hg && per > 0) {
        nxt[u] = ld_stream(reinterpret_cast<const float4*>(H + (size_t(hh_l) * p.sh + size_t(k_l) * RP) * sc));
        if (++k_l == per) { k_l = 0; ++hh_l; }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const bool ok = done + u < total;  // uniform across the LC lanes of a state row
      float dot = 0.f;
      int hh = hh_c, pp = pr + k_c * RP;
      if (ok) {
        const float dt = dts[hh], dc = dcs[hh], xp = xs[hh * pw + pp];
        float4 nv;  // decay*h + (dt*b)*x  (model/kernels.py:163-171)
        nv.x = fmaf(dc, cur[u].x, (dt * b4.x) * xp);
        nv.y = fmaf(dc, cur[u].y, (dt * b4.y) * xp);
        nv.z = fmaf(dc, cur[u].z, (dt * b4.z) * xp);
        nv.w = fmaf(dc, cur[u].w, (dt * b4.w) * xp);
        st_stream(reinterpret_cast<float4*>(H + (size_t(hh) * p.sh + size_t(k_c) * RP) * sc), nv);
        dot = fmaf(cv.w, nv.w, fmaf(cv.z, nv.z, fmaf(cv.y, nv.y, cv.x * nv.x)));
        if (++k_c == per) { k_c = 0; ++hh_c; }
      }
#pragma unroll
      for (int o = LC / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (ok && c4 == 0) p.out[size_t(row) * p.o_rs + size_t(h0 + hh) * p.sh + p0 + pp] = dot;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) cur[u] = nxt[u];
  }
}

// mLSTM / RetNet, kw/4 = L in {8, 16, 32}: thread (hr, c4) walks state rows
// h = hr, hr+RH, ... of each head in the group; the sum over h closes in shared memory.
template <int L>
__global__ void __launch_bounds__(kThreads, 4) outer_rows_fast(const __grid_constant__ OuterRowsParams p, int HG) {
  pdl_wait();
  const int row = blockIdx.z;
  if (row >= live_rows(p.at.n_dev, p.at.n_host)) return;
  constexpr int RH = kThreads / L, KW = 4 * L;
  const int h0 = blockIdx.y * HG;
  const int hg = min(HG, p.nh - h0);
  const int k0 = blockIdx.x * KW;
  const int tid = threadIdx.x;
  const int c4 = tid % L, hr = tid / L;
  if (p.at.mask && !p.at.mask[row]) {
    for (int i = tid; i < hg * KW; i += kThreads)
      p.out[size_t(row) * p.o_rs + size_t(h0 + i / KW) * p.sk + k0 + i % KW] = 0.0f;
    return;
  }
  const int per = hr < p.sh ? (p.sh - hr + RH - 1) / RH : 0;  // state rows per head for this thread
  float* S = p.at.state + size_t(row_slot(p.at, row)) * p.at.row_stride + (size_t(h0) * p.sh + hr) * p.sk + k0 + c4 * 4;
  const size_t hstride = size_t(p.sh) * p.sk;

  float4 cur[U];
  int hh_l = 0, k_l = 0;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (hh_l < hg && per > 0) {
      cur[u] = ld_stream(reinterpret_cast<const float4*>(S + size_t(hh_l) * hstride + size_t(k_l) * RH * p.sk));
      if (++k_l == per) { k_l = 0; ++hh_l; }
    }
  }
  extern __shared__ __align__(16) float sm[];
  const int qn = (HG * p.sh + 3) & ~3;
  float* qs = sm;                      // [hg][sh]
  float* iks = qs + qn;                // [hg][sh] i * k
  float* vs = iks + qn;                // [hg][KW]
  float* fs = vs + HG * KW;            // [hg]
  float* part = fs + ((HG + 3) & ~3);  // [hg][RH][KW]
  for (int i = tid; i < hg * p.sh; i += kThreads) {
    const int hh = i / p.sh, h = i - hh * p.sh, n = h0 + hh;
    const float ii = p.i ? p.i[size_t(row) * p.i_rs + size_t(n) * p.i_hs] : 1.0f;
    qs[i] = p.q[size_t(row) * p.q_rs + size_t(n) * p.sh + h];
    iks[i] = ii * p.kv[size_t(row) * p.k_rs + size_t(n) * p.sh + h];
  }
  for (int i = tid; i < hg * KW; i += kThreads) {
    const int hh = i / KW, k = i - hh * KW;
    vs[i] = p.v[size_t(row) * p.v_rs + size_t(h0 + hh) * p.sk + k0 + k];
  }
  for (int hh = tid; hh < hg; hh += kThreads) fs[hh] = p.f[size_t(row) * p.f_rs + size_t(h0 + hh) * p.f_hs];
  for (int i = tid; i < hg * RH * KW; i += kThreads) part[i] = 0.0f;
  __syncthreads();

  int hh_c = 0, k_c = 0;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  const int total = hg * per;
  for (int done = 0; done < total; done += U) {
    float4 nxt[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (hh_l < hg && per > 0) {
        nxt[u] = ld_stream(reinterpret_cast<const float4*>(S + size_t(hh_l) * hstride + size_t(k_l) * RH * p.sk));
        if (++k_l == per) { k_l = 0; ++hh_l; }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (done + u < total) {
        const int hh = hh_c, h = hr + k_c * RH;
        const float f = fs[hh], ik = iks[hh * p.sh + h], qh = qs[hh * p.sh + h];
        const float4 v4 = *reinterpret_cast<const float4*>(&vs[hh * KW + c4 * 4]);
        float4 nv;  // f*S + (i*k)*v  (model/kernels.py:143-160)
        nv.x = fmaf(f, cur[u].x, ik * v4.x);
        nv.y = fmaf(f, cur[u].y, ik * v4.y);
        nv.z = fmaf(f, cur[u].z, ik * v4.z);
        nv.w = fmaf(f, cur[u].w, ik * v4.w);
        st_stream(reinterpret_cast<float4*>(S + size_t(hh) * hstride + size_t(k_c) * RH * p.sk), nv);
        acc.x = fmaf(qh, nv.x, acc.x);
        acc.y = fmaf(qh, nv.y, acc.y);
        acc.z = fmaf(qh, nv.z, acc.z);
        acc.w = fmaf(qh, nv.w, acc.w);
        if (++k_c == per) {  // head finished: its partial goes to shared memory
          *reinterpret_cast<float4*>(&part[(hh * RH + hr) * KW + c4 * 4]) = acc;
          acc = make_float4(0.f, 0.f, 0.f, 0.f);
          k_c = 0;
          ++hh_c;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) cur[u] = nxt[u];
  }
  __syncthreads();
  for (int i = tid; i < hg * KW; i += kThreads) {
    const int hh = i / KW, k = i - hh * KW;
    float sum = 0.f;
#pragma unroll 4
    for (int r = 0; r < RH; ++r) sum += part[(hh * RH + r) * KW + k];
    p.out[size_t(row) * p.o_rs + size_t(h0 + hh) * p.sk + k0 + k] = sum;
  }
}

}  // namespace

constexpr int kItems = 2048;  // 16-byte vectors per CTA (8 per thread)

void outer_rows(const OuterRowsParams& p, int rows_max, cudaStream_t s, const LaunchCfg& ln) {
  B2E_CHECK(p.sh > 0 && p.sh <= kMaxSh, kErrInvalid, "outer_rows: head size (contracted axis) must be in 1..512");
  B2E_CHECK(p.sk > 0 && p.sk % 4 == 0, kErrInvalid, "outer_rows: carried axis must be a multiple of 4");
  B2E_CHECK(p.nh > 0 && p.nh <= 65535 && rows_max <= 65535, kErrInvalid, "outer_rows: grid too large");
  B2E_CHECK((reinterpret_cast<uintptr_t>(p.at.state) & 15) == 0 && (p.at.row_stride & 3) == 0, kErrInvalid,
            "outer_rows: state must be 16-byte aligned per row");
  if (rows_max <= 0) return;
  if (outer_rows_bulk_ok(p)) {
    outer_rows_bulk(p, rows_max, s, ln);
    return;
  }
  int kt = std::min(kKT, p.sk);
  // a step of few rows: narrower column tiles, so the launch still covers the SMs
  // (one request at the default dims: 8 heads x 4 tiles of 128 -> 8 x 16 of 32)
  while (kt > 32 && p.sk % kt == 0 && long(p.sk / kt) * p.nh * rows_max < 2L * 148) kt /= 2;
  const int per_head = p.sh * (kt / 4);
  const int L = kt / 4, RH = kThreads / L;
  auto smem_of = [&](int hg) {
    return (2 * ((size_t(hg) * p.sh + 3) & ~size_t(3)) + size_t(hg) * kKT + ((hg + 3) & ~3) + size_t(hg) * RH * kt) * 4;
  };
  const bool narrowed = kt < std::min(kKT, p.sk);  // then one head per CTA, for the same reason
  int HG = (p.sk <= kKT && !narrowed) ? std::max(1, std::min(p.nh, kItems / per_head)) : 1;
  while (HG > 1 && (p.nh % HG || smem_of(HG) > 48 * 1024)) --HG;
  const size_t smem = smem_of(HG);
  B2E_CHECK(smem <= 48 * 1024, kErrInvalid, "outer_rows: head too large for one CTA");
  const bool tiles = p.sk % kt == 0;  // every tile full width
  dim3 grid(ceil_div(p.sk, tiles ? kt : kKT), ceil_div(p.nh, HG), rows_max);
  if (tiles && kt == 128)
    launch_k(ln, outer_rows_fast<32>, grid, dim3(kThreads), smem, s, p, HG);
  else if (tiles && kt == 64)
    launch_k(ln, outer_rows_fast<16>, grid, dim3(kThreads), smem, s, p, HG);
  else if (tiles && kt == 32)
    launch_k(ln, outer_rows_fast<8>, grid, dim3(kThreads), smem, s, p, HG);
  else
    launch_k(ln, outer_rows_kernel, grid, dim3(kThreads), smem, s, p, HG);
  B2E_CUDA(cudaGetLastError());
}

void ssm_cols(const SsmColsParams& p, int rows_max, cudaStream_t s, const LaunchCfg& ln) {
  B2E_CHECK(p.sc > 0 && p.sc % 4 == 0 && p.sc <= 4096, kErrInvalid, "ssm_cols: state width must be a multiple of 4, <= 4096");
  B2E_CHECK(p.sh > 0 && p.nh > 0 && p.nh <= 65535 && rows_max <= 65535, kErrInvalid, "ssm_cols: bad sizes");
  B2E_CHECK((reinterpret_cast<uintptr_t>(p.at.state) & 15) == 0 && (p.at.row_stride & 3) == 0, kErrInvalid,
            "ssm_cols: state must be 16-byte aligned per row");
  if (rows_max <= 0) return;
  if (ssm_cols_bulk_ok(p)) {
    ssm_cols_bulk(p, rows_max, s, ln);
    return;
  }
  const int LC = p.sc / 4;
  const int PT = std::min(p.sh, std::max(1, kItems / LC));
  auto smem_of = [&](int hg) {
    return (2 * size_t(p.sc) + 2 * ((hg + 3) & ~3) + ((size_t(hg) * PT + 3) & ~size_t(3)) + size_t(hg) * PT * LC) * 4;
  };
  int HG = PT == p.sh ? std::max(1, std::min(p.nh, kItems / (PT * LC))) : 1;
  while (HG > 1 && (p.nh % HG || smem_of(HG) > 48 * 1024)) --HG;
  const size_t smem = smem_of(HG);
  B2E_CHECK(smem <= 48 * 1024, kErrInvalid, "ssm_cols: state row too wide for one CTA");
  dim3 grid(ceil_div(p.sh, PT), ceil_div(p.nh, HG), rows_max);
  const bool aligned_bc = (reinterpret_cast<uintptr_t>(p.b) & 15) == 0 && (reinterpret_cast<uintptr_t>(p.c) & 15) == 0 &&
                          p.b_rs % 4 == 0 && p.c_rs % 4 == 0;
  if (aligned_bc && LC == 32)
    launch_k(ln, ssm_cols_fast<32>, grid, dim3(kThreads), smem, s, p, PT, HG);
  else if (aligned_bc && LC == 16)
    launch_k(ln, ssm_cols_fast<16>, grid, dim3(kThreads), smem, s, p, PT, HG);
  else if (aligned_bc && LC == 8)
    launch_k(ln, ssm_cols_fast<8>, grid, dim3(kThreads), smem, s, p, PT, HG);
  else
    launch_k(ln, ssm_cols_kernel, grid, dim3(kThreads), smem, s, p, PT, HG);
  B2E_CUDA(cudaGetLastError());
}

}  // namespace b2e
