// SIMT projection GEMMs for sm_100a (see gemm.cuh for the semantics).
//
// Two kernels:
//  * gemm_tiled: 64x64 output tile per CTA, 16-deep K slices through shared
//    memory with a register prefetch of the next slice, 4x4 outputs per thread.
//    f32 FMA arithmetic; each 16-deep slice is summed into a fresh partial that
//    joins the running sum through Kahan's compensated addition, so the error of
//    a long dot product (K = 2048 at the default dims) grows like that of 16
//    terms rather than of K.
//  * gemm_skinny: M <= 16 rows. Weight-bound: each warp streams whole W rows with
//    128-bit loads and keeps one accumulator per live row; this is the path a
//    single request takes, where the step is a chain of GEMVs over the weights.
#include "gemm.cuh"

#include <algorithm>

namespace b2e {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, TPB = 256;

template <int T>
__device__ __forceinline__ float4 load4_vec(const void* base, size_t idx) {
  if constexpr (T == kF32) {
    return __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx));
  } else {
    using L = typename LowP<T>::type;
    uint2 raw = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const L*>(base) + idx));
    L v[4];
    *reinterpret_cast<uint2*>(v) = raw;
    float4 r;
    if constexpr (T == kBF16) {
      r.x = __bfloat162float(v[0]); r.y = __bfloat162float(v[1]);
      r.z = __bfloat162float(v[2]); r.w = __bfloat162float(v[3]);
    } else {
      r.x = __half2float(v[0]); r.y = __half2float(v[1]);
      r.z = __half2float(v[2]); r.w = __half2float(v[3]);
    }
    return r;
  }
}

template <int T>
__device__ __forceinline__ float load1(const void* base, size_t idx) {
  return LowP<T>::load(base, idx);
}

// Load 4 consecutive K elements of one row, zero outside [0, rows) x [0, K).
template <int T>
__device__ __forceinline__ float4 load_row4(const void* base, int ld, int row, int rows, int k, int K, bool vec) {
  float4 r = make_float4(0.f, 0.f, 0.f, 0.f);
  if (row >= rows) return r;
  const size_t off = size_t(row) * ld + k;
  if (vec && k + 3 < K) return load4_vec<T>(base, off);
  if (k + 0 < K) r.x = load1<T>(base, off + 0);
  if (k + 1 < K) r.y = load1<T>(base, off + 1);
  if (k + 2 < K) r.z = load1<T>(base, off + 2);
  if (k + 3 < K) r.w = load1<T>(base, off + 3);
  return r;
}

template <int WT>
__device__ __forceinline__ float4 round4(float4 v) {
  v.x = LowP<WT>::round(v.x); v.y = LowP<WT>::round(v.y);
  v.z = LowP<WT>::round(v.z); v.w = LowP<WT>::round(v.w);
  return v;
}

template <int WT>
__device__ __forceinline__ float epilogue(const GemmParams& p, const GemmGroup& g, float acc, int m, int n) {
  float v = acc;
  if (g.bias) v += load_as(p.bias_type, g.bias, n);
  if (p.round_out) v = LowP<WT>::round(v);
  if (p.act == kActRelu) v = fmaxf(v, 0.0f);
  if (g.R) v += g.R[size_t(m) * p.ldr + n];
  return v;
}

template <int AT, int WT>
__global__ void __launch_bounds__(TPB) gemm_tiled(const __grid_constant__ GemmParams p, bool vec_a, bool vec_w) {
  pdl_wait();
  const GemmGroup& g = p.g[blockIdx.z];
  const int M = live_rows(p.M_dev, p.M_max);
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  if (m0 >= M) return;

  __shared__ float As[2][BK][BM + 4];
  __shared__ float Ws[2][BK][BN + 4];

  const int tid = threadIdx.x;
  const int lr = tid >> 2, lk = (tid & 3) * 4;  // loader: row, k offset
  const int tx = tid & 15, ty = tid >> 4;       // compute: cols 4tx.., rows ty+16i
  const bool round_a = (AT == kF32 && WT != kF32);

  float acc[4][4], cmp[4][4];  // running sums and their Kahan compensations
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = cmp[i][j] = 0.f;

  auto fetch = [&](int k0, float4& a, float4& w) {
    a = load_row4<AT>(g.A, p.lda, m0 + lr, M, k0 + lk, p.K, vec_a);
    if (round_a) a = round4<WT>(a);
    w = load_row4<WT>(g.W, p.ldw, n0 + lr, p.N, k0 + lk, p.K, vec_w);
  };
  auto stash = [&](int buf, const float4& a, const float4& w) {
    As[buf][lk + 0][lr] = a.x; As[buf][lk + 1][lr] = a.y;
    As[buf][lk + 2][lr] = a.z; As[buf][lk + 3][lr] = a.w;
    Ws[buf][lk + 0][lr] = w.x; Ws[buf][lk + 1][lr] = w.y;
    Ws[buf][lk + 2][lr] = w.z; Ws[buf][lk + 3][lr] = w.w;
  };

  float4 ra, rw;
  fetch(0, ra, rw);
  stash(0, ra, rw);
  __syncthreads();
  int buf = 0;
  for (int k0 = 0; k0 < p.K; k0 += BK) {
    const bool more = k0 + BK < p.K;
    if (more) fetch(k0 + BK, ra, rw);
    float part[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) part[i][j] = 0.f;
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[buf][kk][ty + 16 * i];
      const float4 w = *reinterpret_cast<const float4*>(&Ws[buf][kk][tx * 4]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        part[i][0] = fmaf(a[i], w.x, part[i][0]);
        part[i][1] = fmaf(a[i], w.y, part[i][1]);
        part[i][2] = fmaf(a[i], w.z, part[i][2]);
        part[i][3] = fmaf(a[i], w.w, part[i][3]);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {  // Kahan: acc + part, the lost low part kept in cmp
        const float y = part[i][j] - cmp[i][j];
        const float t = acc[i][j] + y;
        cmp[i][j] = (t - acc[i][j]) - y;
        acc[i][j] = t;
      }
    if (more) {
      stash(buf ^ 1, ra, rw);
      __syncthreads();
      buf ^= 1;
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = m0 + ty + 16 * i;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n >= p.N) continue;
      const float v = epilogue<WT>(p, g, acc[i][j], m, n);
      if (g.C) g.C[size_t(m) * p.ldc + n] = v;
      if (g.C_lp) store_as(WT == kF32 ? kF32 : WT, g.C_lp, size_t(m) * p.ldc_lp + n, v);
    }
  }
}

// U consecutive 128-wide K steps of one W row at lane offset k: the U weight
// loads are issued together, then each row's accumulator takes the steps in
// increasing k (the same order of fmas whatever U is).
template <int AT, int WT, int MM, int U>
__device__ __forceinline__ void skinny_steps(const GemmParams& p, const GemmGroup& g, size_t wrow, int k, int M,
                                             float (&acc)[MM]) {
  constexpr bool round_a = (AT == kF32 && WT != kF32);
  float4 w[U];
#pragma unroll
  for (int u = 0; u < U; ++u) w[u] = load4_vec<WT>(g.W, wrow + k + u * 128);
#pragma unroll
  for (int r = 0; r < MM; ++r) {
    if (r < M) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float4 a = load4_vec<AT>(g.A, size_t(r) * p.lda + k + u * 128);
        if (round_a) a = round4<WT>(a);
        acc[r] = fmaf(a.x, w[u].x, acc[r]);
        acc[r] = fmaf(a.y, w[u].y, acc[r]);
        acc[r] = fmaf(a.z, w[u].z, acc[r]);
        acc[r] = fmaf(a.w, w[u].w, acc[r]);
      }
    }
  }
}

// One warp per output column; MM = accumulators per lane (>= live rows).
template <int AT, int WT, int MM>
__global__ void __launch_bounds__(256) gemm_skinny(const __grid_constant__ GemmParams p, bool vec) {
  pdl_wait();
  const GemmGroup& g = p.g[blockIdx.y];
  const int M = min(live_rows(p.M_dev, p.M_max), MM);
  if (M <= 0) return;
  const int lane = threadIdx.x & 31;
  const int warps = blockDim.x >> 5;
  const int gw = blockIdx.x * warps + (threadIdx.x >> 5);
  const int stride = gridDim.x * warps;
  const bool round_a = (AT == kF32 && WT != kF32);

  for (int n = gw; n < p.N; n += stride) {
    float acc[MM];
#pragma unroll
    for (int r = 0; r < MM; ++r) acc[r] = 0.f;
    const size_t wrow = size_t(n) * p.ldw;
    if (vec) {
      // 4 elements per lane per step: 16 steps in flight (a 2048-wide row in
      // one round trip to memory), then 4, then 1
      int k = lane * 4;
      for (; k + 15 * 128 + 3 < p.K; k += 16 * 128) skinny_steps<AT, WT, MM, 16>(p, g, wrow, k, M, acc);
      for (; k + 3 * 128 + 3 < p.K; k += 4 * 128) skinny_steps<AT, WT, MM, 4>(p, g, wrow, k, M, acc);
      for (; k + 3 < p.K; k += 128) skinny_steps<AT, WT, MM, 1>(p, g, wrow, k, M, acc);
    } else {
      for (int k = lane; k < p.K; k += 32) {
        const float w = load1<WT>(g.W, wrow + k);
#pragma unroll
        for (int r = 0; r < MM; ++r) {
          if (r < M) {
            float a = load1<AT>(g.A, size_t(r) * p.lda + k);
            if (round_a) a = LowP<WT>::round(a);
            acc[r] = fmaf(a, w, acc[r]);
          }
        }
      }
    }
#pragma unroll
    for (int r = 0; r < MM; ++r) acc[r] = warp_sum(acc[r]);
    if (lane < M) {
      float mine = 0.f;
#pragma unroll
      for (int r = 0; r < MM; ++r)
        if (r == lane) mine = acc[r];
      const float v = epilogue<WT>(p, g, mine, lane, n);
      if (g.C) g.C[size_t(lane) * p.ldc + n] = v;
      if (g.C_lp) store_as(WT, g.C_lp, size_t(lane) * p.ldc_lp + n, v);
    }
  }
}

// fp32 projections with few outputs (N <= NN: Mamba2's dt_proj, the mLSTM
// input/forget gate projections): one warp per kNarrowRows rows computes every
// output; each lane accumulates its 4-wide K slices against all NN W rows (W
// stays in L1; rows n >= N read row N-1 and are not stored), then a butterfly
// sum closes the dot products across the warp. The next slice of A is loaded
// while the current one is multiplied.
constexpr int kNarrowRows = 2;

template <int NN>
__global__ void __launch_bounds__(256) gemm_narrow(const __grid_constant__ GemmParams p) {
  pdl_wait();
  const GemmGroup& g = p.g[0];
  const int M = live_rows(p.M_dev, p.M_max);
  const int lane = threadIdx.x & 31;
  const int r0 = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * kNarrowRows;
  if (r0 >= M) return;  // warp-uniform
  const float* A = static_cast<const float*>(g.A);
  const float* W = static_cast<const float*>(g.W);
  const float* arow[kNarrowRows];
#pragma unroll
  for (int i = 0; i < kNarrowRows; ++i) arow[i] = A + size_t(min(r0 + i, M - 1)) * p.lda;
  const float* wrow[NN];
#pragma unroll
  for (int n = 0; n < NN; ++n) wrow[n] = W + size_t(min(n, p.N - 1)) * p.ldw;
  float acc[kNarrowRows][NN];
#pragma unroll
  for (int i = 0; i < kNarrowRows; ++i)
#pragma unroll
    for (int n = 0; n < NN; ++n) acc[i][n] = 0.f;
  int k = lane * 4;
  float4 a[kNarrowRows];
#pragma unroll
  for (int i = 0; i < kNarrowRows; ++i)
    a[i] = k < p.K ? *reinterpret_cast<const float4*>(arow[i] + k) : make_float4(0.f, 0.f, 0.f, 0.f);
  for (; k < p.K; k += 128) {
    float4 an[kNarrowRows];
    const int kn = k + 128;
#pragma unroll
    for (int i = 0; i < kNarrowRows; ++i)
      an[i] = kn < p.K ? *reinterpret_cast<const float4*>(arow[i] + kn) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int n = 0; n < NN; ++n) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(wrow[n] + k));
#pragma unroll
      for (int i = 0; i < kNarrowRows; ++i)
        acc[i][n] = fmaf(a[i].w, w.w, fmaf(a[i].z, w.z, fmaf(a[i].y, w.y, fmaf(a[i].x, w.x, acc[i][n]))));
    }
#pragma unroll
    for (int i = 0; i < kNarrowRows; ++i) a[i] = an[i];
  }
#pragma unroll
  for (int i = 0; i < kNarrowRows; ++i)
#pragma unroll
    for (int n = 0; n < NN; ++n) acc[i][n] = warp_sum(acc[i][n]);
  // lane (i * NN + n) % 32 writes output (row r0 + i, column n)
#pragma unroll
  for (int i = 0; i < kNarrowRows; ++i)
#pragma unroll
    for (int n = 0; n < NN; ++n) {
      if ((i * NN + n) % 32 != lane || n >= p.N || r0 + i >= M) continue;
      const int m = r0 + i;
      const float v = epilogue<kF32>(p, g, acc[i][n], m, n);
      if (g.C) g.C[size_t(m) * p.ldc + n] = v;
      if (g.C_lp) store_as(kF32, g.C_lp, size_t(m) * p.ldc_lp + n, v);
    }
}

// Same problem with W staged once per CTA in shared memory (when it fits): a
// persistent grid of warps walks the rows, each lane streaming its 4-wide K
// slices of A and reading W from shared memory, so the A stream cannot evict W.
constexpr size_t kNarrowSmemMax = 100 * 1024;

template <int NN>
__global__ void __launch_bounds__(256) gemm_narrow_smem(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(16) float ws[];  // [N][K]
  const float* W = static_cast<const float*>(p.g[0].W);
  const int K4 = p.K >> 2, N = p.N;
  // weights (no predecessor writes them), eight 16-byte loads in flight per thread
  for (int i0 = threadIdx.x; i0 < N * K4; i0 += blockDim.x * 8) {
    float4 t[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + j * blockDim.x, n = i / K4;
      if (i < N * K4) t[j] = __ldg(reinterpret_cast<const float4*>(W + size_t(n) * p.ldw) + (i - n * K4));
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (i0 + j * blockDim.x < N * K4) reinterpret_cast<float4*>(ws)[i0 + j * blockDim.x] = t[j];
  }
  pdl_wait();
  const int M = live_rows(p.M_dev, p.M_max);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const float* A = static_cast<const float*>(p.g[0].A);
  const int lda = p.lda;
  const float4* ws4 = reinterpret_cast<const float4*>(ws);
  constexpr int R = 2, U = 4;  // rows per warp, K iterations whose loads go out together
  const int wstride = gridDim.x * (blockDim.x >> 5) * R;
  for (int m = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * R; m < M; m += wstride) {
    float acc[R][NN];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int n = 0; n < NN; ++n) acc[r][n] = 0.f;
    const float4* a4[R];
#pragma unroll
    for (int r = 0; r < R; ++r) a4[r] = reinterpret_cast<const float4*>(A + size_t(min(m + r, M - 1)) * lda);
    for (int kc = lane; kc < K4; kc += 32 * U) {
      float4 a[R][U];
#pragma unroll
      for (int j = 0; j < U; ++j)
#pragma unroll
        for (int r = 0; r < R; ++r)
          a[r][j] = kc + 32 * j < K4 ? a4[r][kc + 32 * j] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < U; ++j) {
        const int k4 = min(kc + 32 * j, K4 - 1);  // past K: a is zero
#pragma unroll
        for (int n = 0; n < NN; ++n) {
          const float4 w = ws4[min(n, N - 1) * K4 + k4];
#pragma unroll
          for (int r = 0; r < R; ++r)
            acc[r][n] = fmaf(a[r][j].w, w.w, fmaf(a[r][j].z, w.z, fmaf(a[r][j].y, w.y, fmaf(a[r][j].x, w.x, acc[r][n]))));
        }
      }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int n = 0; n < NN; ++n) acc[r][n] = warp_sum(acc[r][n]);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int n = 0; n < NN; ++n)
        if (r * NN + n == lane && n < N && m + r < M) {
          const GemmGroup& g = p.g[0];
          const float v = epilogue<kF32>(p, g, acc[r][n], m + r, n);
          if (g.C) g.C[size_t(m + r) * p.ldc + n] = v;
          if (g.C_lp) store_as(kF32, g.C_lp, size_t(m + r) * p.ldc_lp + n, v);
        }
  }
}

bool narrow_eligible(const GemmParams& p) {
  return p.groups == 1 && p.a_type == kF32 && p.w_type == kF32 && p.N <= 16 && p.M_max > 16 && p.K % 4 == 0 &&
         p.lda % 4 == 0 && p.ldw % 4 == 0 && (reinterpret_cast<uintptr_t>(p.g[0].A) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(p.g[0].W) & 15) == 0;
}

bool aligned(const void* ptr, int bytes) { return (reinterpret_cast<uintptr_t>(ptr) % bytes) == 0; }

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int AT, int WT>
void launch(const GemmParams& p, cudaStream_t s) {
  const int abytes = int(dtype_size(AT)), wbytes = int(dtype_size(WT));
  bool vec_a = (p.K % 4 == 0) && (p.lda % 4 == 0);
  bool vec_w = (p.K % 4 == 0) && (p.ldw % 4 == 0);
  for (int i = 0; i < p.groups; ++i) {
    vec_a = vec_a && aligned(p.g[i].A, 4 * abytes);
    vec_w = vec_w && aligned(p.g[i].W, 4 * wbytes);
  }
  if (p.M_max <= 16) {
    const int warps = 8;
    int blocks = ceil_div(p.N, warps);
    blocks = std::min(blocks, 8 * sm_count());
    dim3 grid(blocks, p.groups);
    const bool vec = vec_a && vec_w;
    if (p.M_max <= 1)
      launch_k(p.ln, gemm_skinny<AT, WT, 1>, grid, dim3(32 * warps), 0, s, p, vec);
    else if (p.M_max <= 2)
      launch_k(p.ln, gemm_skinny<AT, WT, 2>, grid, dim3(32 * warps), 0, s, p, vec);
    else if (p.M_max <= 4)
      launch_k(p.ln, gemm_skinny<AT, WT, 4>, grid, dim3(32 * warps), 0, s, p, vec);
    else if (p.M_max <= 8)
      launch_k(p.ln, gemm_skinny<AT, WT, 8>, grid, dim3(32 * warps), 0, s, p, vec);
    else
      launch_k(p.ln, gemm_skinny<AT, WT, 16>, grid, dim3(32 * warps), 0, s, p, vec);
  } else {
    dim3 grid(ceil_div(p.N, BN), ceil_div(p.M_max, BM), p.groups);
    launch_k(p.ln, gemm_tiled<AT, WT>, grid, dim3(TPB), 0, s, p, vec_a, vec_w);
  }
}

}  // namespace

void gemm_simt_init() {
  B2E_CUDA(cudaFuncSetAttribute(gemm_narrow_smem<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kNarrowSmemMax)));
  B2E_CUDA(cudaFuncSetAttribute(gemm_narrow_smem<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(kNarrowSmemMax)));
}

void gemm(const GemmParams& p, cudaStream_t s) {
  B2E_CHECK(p.groups >= 1 && p.groups <= kMaxGroups, kErrInternal, "gemm: bad group count");
  B2E_CHECK(p.M_max > 0 && p.N > 0 && p.K > 0, kErrInternal, "gemm: empty problem");
  B2E_CHECK(p.M_max <= 65535 * BM, kErrInternal, "gemm: too many rows");
  if (gemm_tc_eligible(p)) {
    gemm_tc(p, s);
    return;
  }
  if (narrow_eligible(p) && size_t(p.N) * p.K * 4 <= kNarrowSmemMax) {
    const size_t smem = size_t(p.N) * p.K * 4;
    const int blocks = std::min(ceil_div(p.M_max, 16), 2 * sm_count());
    if (p.N <= 8)
      launch_k(p.ln, gemm_narrow_smem<8>, dim3(blocks), dim3(256), smem, s, p);
    else
      launch_k(p.ln, gemm_narrow_smem<16>, dim3(blocks), dim3(256), smem, s, p);
    return;
  }
  if (narrow_eligible(p)) {
    const int blocks = ceil_div(p.M_max, 8 * kNarrowRows);
    if (p.N <= 8)
      launch_k(p.ln, gemm_narrow<8>, dim3(blocks), dim3(256), 0, s, p);
    else
      launch_k(p.ln, gemm_narrow<16>, dim3(blocks), dim3(256), 0, s, p);
    return;
  }
  const int a = p.a_type, w = p.w_type;
  if (w == kF32) {
    B2E_CHECK(a == kF32, kErrInternal, "gemm: f32 weights need f32 activations");
    launch<kF32, kF32>(p, s);
  } else if (w == kBF16) {
    if (a == kF32) launch<kF32, kBF16>(p, s);
    else if (a == kBF16) launch<kBF16, kBF16>(p, s);
    else throw Error(kErrInternal, "gemm: activation/weight type mismatch");
  } else if (w == kF16) {
    if (a == kF32) launch<kF32, kF16>(p, s);
    else if (a == kF16) launch<kF16, kF16>(p, s);
    else throw Error(kErrInternal, "gemm: activation/weight type mismatch");
  } else {
    throw Error(kErrInternal, "gemm: unknown weight type");
  }
  B2E_CUDA(cudaGetLastError());
}

}  // namespace b2e
