// State-streaming recurrent steps (see cells.cuh).
//
// Memory plan: one CTA owns one (row, head, tile) of the state. Every thread
// moves 16-byte vectors with evict-first loads/stores and keeps four of them in
// flight before it computes, so a 148-SM part has ~100 KB of loads outstanding
// per SM - enough to cover HBM latency at full bandwidth. The small per-row
// operands (q, i*k, v or dt*b, c, x) are staged once in shared memory.
#include "cells.cuh"

#include <algorithm>

namespace b2e {
namespace {

constexpr int kThreads = 256;
constexpr int kMaxSh = 512;   // largest contracted/carried head axis kept in smem
constexpr int kKT = 128;      // k-columns per CTA in outer_rows
constexpr int kPart = 1024;   // partial-sum slots per CTA

__device__ __forceinline__ int row_slot(const RowAddr& a, int row) { return a.slots ? a.slots[row] : row; }

__global__ void __launch_bounds__(kThreads) outer_rows_kernel(const __grid_constant__ OuterRowsParams p) {
  const int row = blockIdx.z;
  if (row >= live_rows(p.at.n_dev, p.at.n_host)) return;
  const int n = blockIdx.y;
  const int k0 = blockIdx.x * kKT;
  const int kw = min(kKT, p.sk - k0);
  const int tid = threadIdx.x;
  float* out = p.out + size_t(row) * p.o_rs + size_t(n) * p.sk + k0;

  if (p.at.mask && !p.at.mask[row]) {  // idle: state untouched, output zero
    for (int k = tid; k < kw; k += kThreads) out[k] = 0.0f;
    return;
  }

  __shared__ float qs[kMaxSh], iks[kMaxSh];
  __shared__ __align__(16) float vs[kKT];
  __shared__ __align__(16) float part[kPart];

  const float f = p.f[size_t(row) * p.f_rs + size_t(n) * p.f_hs];
  const float ii = p.i ? p.i[size_t(row) * p.i_rs + size_t(n) * p.i_hs] : 1.0f;
  for (int h = tid; h < p.sh; h += kThreads) {
    qs[h] = p.q[size_t(row) * p.q_rs + size_t(n) * p.sh + h];
    iks[h] = ii * p.kv[size_t(row) * p.k_rs + size_t(n) * p.sh + h];
  }
  for (int k = tid; k < kw; k += kThreads) vs[k] = p.v[size_t(row) * p.v_rs + size_t(n) * p.sk + k0 + k];
  __syncthreads();

  const int L = kw >> 2;          // float4 lanes across the tile's columns
  const int RH = kThreads / L;    // state rows processed per pass
  const int c4 = tid % L, hr = tid / L;
  float* S = p.at.state + size_t(row_slot(p.at, row)) * p.at.row_stride + size_t(n) * p.sh * p.sk + k0 + c4 * 4;

  if (hr < RH) {
    const float4 v4 = *reinterpret_cast<const float4*>(&vs[c4 * 4]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int h0 = hr; h0 < p.sh; h0 += 4 * RH) {
      float4 s[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int h = h0 + u * RH;
        if (h < p.sh) s[u] = ld_stream(reinterpret_cast<const float4*>(S + size_t(h) * p.sk));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int h = h0 + u * RH;
        if (h < p.sh) {
          const float ik = iks[h], qh = qs[h];
          float4 nv;
          nv.x = fmaf(f, s[u].x, ik * v4.x);
          nv.y = fmaf(f, s[u].y, ik * v4.y);
          nv.z = fmaf(f, s[u].z, ik * v4.z);
          nv.w = fmaf(f, s[u].w, ik * v4.w);
          st_stream(reinterpret_cast<float4*>(S + size_t(h) * p.sk), nv);
          acc.x = fmaf(qh, nv.x, acc.x);
          acc.y = fmaf(qh, nv.y, acc.y);
          acc.z = fmaf(qh, nv.z, acc.z);
          acc.w = fmaf(qh, nv.w, acc.w);
        }
      }
    }
    *reinterpret_cast<float4*>(&part[hr * kw + c4 * 4]) = acc;
  }
  __syncthreads();
  for (int k = tid; k < kw; k += kThreads) {
    float sum = 0.f;
    for (int r = 0; r < RH; ++r) sum += part[r * kw + k];
    out[k] = sum;
  }
}

__global__ void __launch_bounds__(kThreads) ssm_cols_kernel(const __grid_constant__ SsmColsParams p, int PT) {
  const int row = blockIdx.z;
  if (row >= live_rows(p.at.n_dev, p.at.n_host)) return;
  const int n = blockIdx.y;
  const int p0 = blockIdx.x * PT;
  const int pw = min(PT, p.sh - p0);
  const int tid = threadIdx.x;
  float* out = p.out + size_t(row) * p.o_rs + size_t(n) * p.sh + p0;

  if (p.at.mask && !p.at.mask[row]) {
    for (int i = tid; i < pw; i += kThreads) out[i] = 0.0f;
    return;
  }

  extern __shared__ __align__(16) float sm[];
  float* bsd = sm;              // dt * b[c]
  float* cs = bsd + p.sc;       // c[c]
  float* xs = cs + p.sc;        // x[p]
  float* part = xs + ((PT + 3) & ~3);

  const float dt = p.dt[size_t(row) * p.dt_rs + n];
  const float dc = p.decay[size_t(row) * p.dc_rs + n];
  for (int c = tid; c < p.sc; c += kThreads) {
    bsd[c] = dt * p.b[size_t(row) * p.b_rs + c];
    cs[c] = p.c[size_t(row) * p.c_rs + c];
  }
  for (int i = tid; i < pw; i += kThreads) xs[i] = p.x[size_t(row) * p.x_rs + size_t(n) * p.sh + p0 + i];
  __syncthreads();

  const int LC = p.sc >> 2;
  const int items = pw * LC;
  float* H = p.at.state + size_t(row_slot(p.at, row)) * p.at.row_stride + (size_t(n) * p.sh + p0) * p.sc;
  for (int it0 = tid; it0 < items; it0 += 4 * kThreads) {
    float4 s[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int it = it0 + u * kThreads;
      if (it < items) s[u] = ld_stream(reinterpret_cast<const float4*>(H + size_t(it) * 4));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int it = it0 + u * kThreads;
      if (it < items) {
        const int pi = it / LC, c4 = it - pi * LC;
        const float xp = xs[pi];
        const float4 bb = *reinterpret_cast<const float4*>(&bsd[c4 * 4]);
        const float4 cc = *reinterpret_cast<const float4*>(&cs[c4 * 4]);
        float4 nv;
        nv.x = fmaf(dc, s[u].x, bb.x * xp);
        nv.y = fmaf(dc, s[u].y, bb.y * xp);
        nv.z = fmaf(dc, s[u].z, bb.z * xp);
        nv.w = fmaf(dc, s[u].w, bb.w * xp);
        st_stream(reinterpret_cast<float4*>(H + size_t(it) * 4), nv);
        part[it] = fmaf(cc.w, nv.w, fmaf(cc.z, nv.z, fmaf(cc.y, nv.y, cc.x * nv.x)));
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < pw; i += kThreads) {
    float sum = 0.f;
    for (int c4 = 0; c4 < LC; ++c4) sum += part[i * LC + c4];
    out[i] = sum;
  }
}

}  // namespace

void outer_rows(const OuterRowsParams& p, int rows_max, cudaStream_t s) {
  B2E_CHECK(p.sh > 0 && p.sh <= kMaxSh, kErrInvalid, "outer_rows: head size (contracted axis) must be in 1..512");
  B2E_CHECK(p.sk > 0 && p.sk % 4 == 0, kErrInvalid, "outer_rows: carried axis must be a multiple of 4");
  B2E_CHECK(p.nh > 0 && p.nh <= 65535 && rows_max <= 65535, kErrInvalid, "outer_rows: grid too large");
  B2E_CHECK((reinterpret_cast<uintptr_t>(p.at.state) & 15) == 0 && (p.at.row_stride & 3) == 0, kErrInvalid,
            "outer_rows: state must be 16-byte aligned per row");
  if (rows_max <= 0) return;
  dim3 grid(ceil_div(p.sk, kKT), p.nh, rows_max);
  outer_rows_kernel<<<grid, kThreads, 0, s>>>(p);
  B2E_CUDA(cudaGetLastError());
}

void ssm_cols(const SsmColsParams& p, int rows_max, cudaStream_t s) {
  B2E_CHECK(p.sc > 0 && p.sc % 4 == 0 && p.sc <= 4096, kErrInvalid, "ssm_cols: state width must be a multiple of 4, <= 4096");
  B2E_CHECK(p.sh > 0 && p.nh > 0 && p.nh <= 65535 && rows_max <= 65535, kErrInvalid, "ssm_cols: bad sizes");
  B2E_CHECK((reinterpret_cast<uintptr_t>(p.at.state) & 15) == 0 && (p.at.row_stride & 3) == 0, kErrInvalid,
            "ssm_cols: state must be 16-byte aligned per row");
  if (rows_max <= 0) return;
  const int LC = p.sc / 4;
  int PT = std::max(1, kPart / LC);
  PT = std::min(PT, p.sh);
  const size_t smem = (2 * size_t(p.sc) + ((PT + 3) & ~3) + size_t(PT) * LC) * sizeof(float);
  dim3 grid(ceil_div(p.sh, PT), p.nh, rows_max);
  ssm_cols_kernel<<<grid, kThreads, smem, s>>>(p, PT);
  B2E_CUDA(cudaGetLastError());
}

}  // namespace b2e
