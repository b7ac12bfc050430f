// tcgen05 (5th-generation tensor core) GEMM for the CastLinear projections.
//
// C[m, n] = epilogue( sum_k A[m, k] * W[n, k] ), A and W both bf16 (or both f16)
// in global memory, f32 accumulation in tensor memory. One CTA computes one
// 128 x BN output tile (BN = 128, or 256 so that a tile holds whole rows):
//   warp 0     one thread issues TMA loads of A and W tiles (rows x 64 K,
//              128-byte swizzle) into a 3-stage shared-memory ring;
//   warp 1     allocates BN TMEM columns; one thread issues tcgen05.mma
//              (M=128, N=BN, K=16 per instruction) and commits each stage back
//              to the producer and the finished accumulator to the epilogue;
//   warps 2-5  epilogue, in two phases. Phase 1: each warp reads its 32-lane
//              TMEM quadrant (one thread per row) with tcgen05.ld, applies bias,
//              CastLinear rounding and activation, and stages the tile in the
//              now idle operand ring. Phase 2: each warp takes whole rows (lane
//              = 16-byte column unit) and writes them with row-contiguous
//              stores, adding the residual; optional row work (RowEpi: LayerNorm,
//              a second residual, the next RMSNorm, a dot product) runs here with
//              warp-shuffle reductions.
// Every mbarrier wait is bounded: past ~1 s the kernel records an error code,
// stops issuing work, waits (bounded) for what it issued, frees its TMEM and
// returns. TMA loads here never use cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gemm.cuh"

namespace b2e {
namespace {

constexpr int BM = 128, BK = 64, STAGES = 3, THREADS = 192;
constexpr uint32_t TILE_A = BM * BK * 2;
constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz

template <int BN>
struct Cfg {
  static constexpr uint32_t TILE_B = BN * BK * 2;
  static constexpr uint32_t TMEM_COLS = BN;
  static constexpr size_t SMEM = size_t(STAGES) * (TILE_A + TILE_B) + 1024 + 256;
  static_assert(size_t(BM) * BN * 4 <= size_t(STAGES) * (TILE_A + TILE_B), "epilogue stage must fit the ring");
};

enum TcError : int { kTcTimeoutProducer = 101, kTcTimeoutMma = 102, kTcTimeoutEpilogue = 103 };

struct TcEpi {
  const void* bias;
  int bias_type;
  float* C;
  int ldc;
  void* C_lp;
  int ldc_lp;
  const float* R;
  int ldr;
  int M_max;
  const int* M_dev;
  int N, K;
  int lp;  // kBF16 or kF16: operand type and CastLinear rounding type
  int round_out, act;
  int* err;
  int vec;  // every row start of bias/R/C/C_lp (and RowEpi buffers) is 16-byte (f32) / 8-byte (low) aligned
  RowEpi row;
  int row_on;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: true when the phase completed, false on timeout or abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag) {
  const long long t0 = clock64();
  while (!mbar_try(b, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row swizzle atoms 1024 bytes apart (SBO), sm100 version bit.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= uint64_t((addr & 0x3FFFF) >> 4);      // start address
  d |= uint64_t(1) << 16;                    // leading byte offset (unused for swizzled K-major)
  d |= uint64_t(1024 >> 4) << 32;            // stride byte offset
  d |= uint64_t(1) << 46;                    // descriptor version (sm100)
  d |= uint64_t(2) << 61;                    // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: f32 accumulator, A/B type, both K-major.
__host__ __device__ constexpr uint32_t instr_desc(int lp, int bn) {
  const uint32_t ab = lp == kBF16 ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | (uint32_t(bn >> 3) << 17) | (uint32_t(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// 4 consecutive values of a vector of type t (f32, bf16 or f16), 16/8-byte aligned.
__device__ __forceinline__ float4 load4(int t, const void* p, int i) {
  if (t == kF32) return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
  const uint2 raw = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + i);
  float4 r;
  if (t == kBF16) {
    r.x = __uint_as_float(raw.x << 16); r.y = __uint_as_float(raw.x & 0xffff0000u);
    r.z = __uint_as_float(raw.y << 16); r.w = __uint_as_float(raw.y & 0xffff0000u);
  } else {
    const __half2 a = *reinterpret_cast<const __half2*>(&raw.x), b = *reinterpret_cast<const __half2*>(&raw.y);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    r = make_float4(fa.x, fa.y, fb.x, fb.y);
  }
  return r;
}

// Round 4 floats to the low type and back (CastLinear's output rounding), two at a time.
__device__ __forceinline__ float4 round4_lp(int t, float4 x) {
  if (t == kBF16) {
    const float2 a = __bfloat1622float2(__floats2bfloat162_rn(x.x, x.y));
    const float2 b = __bfloat1622float2(__floats2bfloat162_rn(x.z, x.w));
    return make_float4(a.x, a.y, b.x, b.y);
  }
  const float2 a = __half22float2(__floats2half2_rn(x.x, x.y));
  const float2 b = __half22float2(__floats2half2_rn(x.z, x.w));
  return make_float4(a.x, a.y, b.x, b.y);
}

// Store 4 floats as the low type (8 bytes, aligned).
__device__ __forceinline__ void store4_lp(int t, void* p, size_t i, float4 x) {
  uint2 raw;
  if (t == kBF16) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x.x, x.y), b = __floats2bfloat162_rn(x.z, x.w);
    raw.x = *reinterpret_cast<const uint32_t*>(&a);
    raw.y = *reinterpret_cast<const uint32_t*>(&b);
  } else {
    const __half2 a = __floats2half2_rn(x.x, x.y), b = __floats2half2_rn(x.z, x.w);
    raw.x = *reinterpret_cast<const uint32_t*>(&a);
    raw.y = *reinterpret_cast<const uint32_t*>(&b);
  }
  *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + i) = raw;
}

__device__ __forceinline__ float4 f4add(float4 a, float4 b) { return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
__device__ __forceinline__ float f4sum(float4 a) { return (a.x + a.y) + (a.z + a.w); }

template <int BN>
__global__ void __launch_bounds__(THREADS, BN == 128 ? 2 : 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                   const __grid_constant__ TcEpi e) {
  using K = Cfg<BN>;
  constexpr int UPR = BN / 4;    // 16-byte units per tile row
  constexpr int UPL = UPR / 32;  // units per lane in phase 2
  const int M = live_rows(e.M_dev, e.M_max);
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  if (m0 >= M) return;  // whole CTA, before any barrier or TMEM use

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * TILE_A;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + STAGES * K::TILE_B);
  uint64_t* empty = full + STAGES;
  uint64_t* done = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(K::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  const int nkb = (e.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (kb >= STAGES && !mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
          if (!*abort_flag) atomicExch(e.err, kTcTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&full[s], TILE_A + K::TILE_B);
        tma_load_2d(sA + s * TILE_A, &ta, kb * BK, m0, &full[s]);
        tma_load_2d(sB + s * K::TILE_B, &tb, kb * BK, n0, &full[s]);
        ++issued;
      }
      if (*abort_flag) {
        // drain: every load issued lands before the CTA leaves (bounded)
        volatile int never = 0;
        for (int kb = max(0, issued - STAGES); kb < issued; ++kb)
          mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1, &never);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      const uint32_t idesc = instr_desc(e.lp, BN);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag)) {
          if (!*abort_flag) atomicExch(e.err, kTcTimeoutMma);
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a0 = smem_u32(sA + s * TILE_A), b0 = smem_u32(sB + s * K::TILE_B);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)  // K=16 per instruction: +32 bytes inside the swizzled row
          mma_f16(tmem, smem_desc(a0 + k * 32), smem_desc(b0 + k * 32), idesc, (kb | k) != 0);
        mma_commit(&empty[s]);  // frees the stage once these MMAs have read it
      }
      mma_commit(done);  // accumulator complete (covers every MMA issued)
    }
  } else {
    // ---- epilogue: warps 2..5, TMEM lane quadrant = warp % 4
    volatile int never = 0;  // the MMA thread always commits `done`, even after an abort
    const bool ok = mbar_wait(done, 0, &never);
    if (!ok) {
      atomicExch(e.err, kTcTimeoutEpilogue);
      *abort_flag = 1;
    }
    // Both named barriers below are reached by all four epilogue warps whatever
    // happens, so an error path cannot leave a warp waiting; `go` is read once.
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const bool go = ok && !*abort_flag;
    const int q = warp & 3;
    const int m = m0 + q * 32 + lane;
    const bool row_ok = m < M;
    if (go) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (e.vec) {
      // Phase 1: bias, rounding, activation per column; tile to shared memory
      // (the operand ring is idle once `done` fired). 16-byte unit u of tile row
      // r lives at unit u ^ (r & 7): the 32 rows a warp writes fall in distinct
      // bank groups.
      float4* stage = reinterpret_cast<float4*>(sA);  // BM x BN floats
      for (int c0 = 0; go && c0 < BN; c0 += 32) {
        if (n0 + c0 >= e.N) break;  // warp-uniform
        float v[32];
        tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(c0), v);
        const int nb = n0 + c0;
        const int r = q * 32 + lane;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 x = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          if (e.bias && nb + j < e.N) x = f4add(x, load4(e.bias_type, e.bias, nb + j));
          if (e.round_out) x = round4_lp(e.lp, x);
          if (e.act == kActRelu) {
            x.x = fmaxf(x.x, 0.f); x.y = fmaxf(x.y, 0.f); x.z = fmaxf(x.z, 0.f); x.w = fmaxf(x.w, 0.f);
          }
          const int unit = (c0 + j) >> 2;
          stage[r * UPR + (unit ^ (r & 7))] = x;
        }
      }
      // Phase 2: whole rows per warp; lane l owns units l, l+32, ... of a row.
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const RowEpi& re = e.row;
      for (int r = warp - 2; go && r < BM; r += 4) {
        const int mm = m0 + r;
        if (mm >= M) break;  // rows only grow
        float4 x[UPL];
        bool in[UPL];
#pragma unroll
        for (int u = 0; u < UPL; ++u) {
          const int unit = lane + 32 * u;
          const int n = n0 + unit * 4;
          in[u] = n < e.N;
          x[u] = in[u] ? stage[r * UPR + (unit ^ (r & 7))] : make_float4(0.f, 0.f, 0.f, 0.f);
          if (in[u] && e.R) x[u] = f4add(x[u], *reinterpret_cast<const float4*>(e.R + size_t(mm) * e.ldr + n));
        }
        if (e.row_on) {
          const float invN = 1.0f / float(e.N);
          if (re.ln_w) {  // LayerNorm(bias=False): two-pass mean and biased variance
            float s = 0.f;
#pragma unroll
            for (int u = 0; u < UPL; ++u) s += f4sum(x[u]);
            const float mu = warp_sum(s) * invN;
            float q2 = 0.f;
#pragma unroll
            for (int u = 0; u < UPL; ++u)
              if (in[u]) {
                const float4 d = make_float4(x[u].x - mu, x[u].y - mu, x[u].z - mu, x[u].w - mu);
                q2 += f4sum(make_float4(d.x * d.x, d.y * d.y, d.z * d.z, d.w * d.w));
              }
            const float rs = 1.0f / sqrtf(warp_sum(q2) * invN + re.ln_eps);
#pragma unroll
            for (int u = 0; u < UPL; ++u)
              if (in[u]) {
                const int n = n0 + (lane + 32 * u) * 4;
                const float4 w = *reinterpret_cast<const float4*>(re.ln_w + n);
                x[u] = make_float4((x[u].x - mu) * rs * w.x, (x[u].y - mu) * rs * w.y, (x[u].z - mu) * rs * w.z,
                                   (x[u].w - mu) * rs * w.w);
              }
          }
          if (re.R2) {
#pragma unroll
            for (int u = 0; u < UPL; ++u)
              if (in[u])
                x[u] = f4add(x[u], *reinterpret_cast<const float4*>(re.R2 + size_t(mm) * re.ldr2 + n0 + (lane + 32 * u) * 4));
          }
        }
#pragma unroll
        for (int u = 0; u < UPL; ++u)
          if (in[u]) {
            const int n = n0 + (lane + 32 * u) * 4;
            if (e.C) *reinterpret_cast<float4*>(e.C + size_t(mm) * e.ldc + n) = x[u];
            if (e.C_lp) store4_lp(e.lp, e.C_lp, size_t(mm) * e.ldc_lp + n, x[u]);
          }
        if (e.row_on && re.norm_w) {  // nn.RMSNorm of the finished row
          float ss = 0.f;
#pragma unroll
          for (int u = 0; u < UPL; ++u)
            ss += f4sum(make_float4(x[u].x * x[u].x, x[u].y * x[u].y, x[u].z * x[u].z, x[u].w * x[u].w));
          const float inv = 1.0f / sqrtf(warp_sum(ss) * (1.0f / float(e.N)) + re.norm_eps);
#pragma unroll
          for (int u = 0; u < UPL; ++u)
            if (in[u]) {
              const int n = n0 + (lane + 32 * u) * 4;
              const float4 w = *reinterpret_cast<const float4*>(re.norm_w + n);
              const float4 t = make_float4(x[u].x * inv * w.x, x[u].y * inv * w.y, x[u].z * inv * w.z, x[u].w * inv * w.w);
              if (re.T) *reinterpret_cast<float4*>(re.T + size_t(mm) * re.ldt + n) = t;
              if (re.T_lp) store4_lp(e.lp, re.T_lp, size_t(mm) * re.ldt + n, t);
            }
        }
        if (e.row_on && re.dot_w) {  // output_proj: v . w + b
          float d = 0.f;
#pragma unroll
          for (int u = 0; u < UPL; ++u)
            if (in[u]) {
              const float4 w = *reinterpret_cast<const float4*>(re.dot_w + n0 + (lane + 32 * u) * 4);
              d += f4sum(make_float4(x[u].x * w.x, x[u].y * w.y, x[u].z * w.z, x[u].w * w.w));
            }
          d = warp_sum(d);
          if (lane == 0) re.dot_out[size_t(mm) * re.dot_ld + re.dot_col] = d + re.dot_b[0];
        }
      }
    } else {
      for (int c0 = 0; go && c0 < BN; c0 += 32) {
        if (n0 + c0 >= e.N) break;  // warp-uniform
        float v[32];
        tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(c0), v);
        if (!row_ok) continue;
        const int nb = n0 + c0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int n = nb + j;
          if (n >= e.N) continue;
          float x = v[j];
          if (e.bias) x += load_as(e.bias_type, e.bias, n);
          if (e.round_out) x = round_to(e.lp, x);
          if (e.act == kActRelu) x = fmaxf(x, 0.0f);
          if (e.R) x += e.R[size_t(m) * e.ldr + n];
          if (e.C) e.C[size_t(m) * e.ldc + n] = x;
          if (e.C_lp) store_as(e.lp, e.C_lp, size_t(m) * e.ldc_lp + n, x);
        }
      }
    }
  }

  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(K::TMEM_COLS));
  }
}

// ------------------------------------------------------------------ host

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

void make_map(CUtensorMap* m, const void* base, int lp, uint64_t inner, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  auto fn = encode_fn();
  B2E_CHECK(fn != nullptr, kErrCuda, "cuTensorMapEncodeTiled is unavailable");
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {BK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, lp == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  B2E_CHECK(r == CUDA_SUCCESS, kErrCuda, "cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7) == 0; }

template <int BN>
void launch_tc(const GemmParams& p, bool vec, cudaStream_t s) {
  CUtensorMap ta, tb;
  make_map(&ta, p.g[0].A, p.w_type, uint64_t(p.K), uint64_t(p.M_max), uint64_t(p.lda), BM);
  make_map(&tb, p.g[0].W, p.w_type, uint64_t(p.K), uint64_t(p.N), uint64_t(p.ldw), BN);
  const GemmGroup& g = p.g[0];
  TcEpi e{g.bias, p.bias_type, g.C, p.ldc, g.C_lp, p.ldc_lp, g.R, p.ldr, p.M_max, p.M_dev,
          p.N, p.K, p.w_type, p.round_out, p.act, p.err, vec ? 1 : 0, p.row, p.row.active() ? 1 : 0};
  dim3 grid(ceil_div(p.N, BN), ceil_div(p.M_max, BM));
  gemm_tc_kernel<BN><<<grid, THREADS, Cfg<BN>::SMEM, s>>>(ta, tb, e);
  B2E_CUDA(cudaGetLastError());
}

bool row_buffers_ok(const GemmParams& p) {
  const RowEpi& r = p.row;
  return (!r.ln_w || aligned16(r.ln_w)) && (!r.R2 || (aligned16(r.R2) && r.ldr2 % 4 == 0)) &&
         (!r.norm_w || aligned16(r.norm_w)) && (!r.T || (aligned16(r.T) && r.ldt % 4 == 0)) &&
         (!r.T_lp || (aligned8(r.T_lp) && r.ldt % 4 == 0)) &&
         (!r.dot_w || (aligned16(r.dot_w) && r.dot_b && r.dot_out));
}

}  // namespace

void gemm_tc_init() {
  B2E_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg<128>::SMEM)));
  B2E_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(Cfg<256>::SMEM)));
}

bool gemm_tc_eligible(const GemmParams& p) {
  return p.groups == 1 && (p.w_type == kBF16 || p.w_type == kF16) && p.a_type == p.w_type && p.M_max > 16 &&
         p.K % 8 == 0 && p.lda % 8 == 0 && p.ldw % 8 == 0 && p.N % 16 == 0 && aligned16(p.g[0].A) &&
         aligned16(p.g[0].W) && p.err != nullptr && encode_fn() != nullptr;
}

bool gemm_tc_row_eligible(const GemmParams& p) {
  return gemm_tc_eligible(p) && p.N <= 256 && row_buffers_ok(p);
}

void gemm_tc(const GemmParams& p, cudaStream_t s) {
  B2E_CHECK(gemm_tc_eligible(p), kErrInternal, "gemm_tc: problem not eligible");
  const GemmGroup& g = p.g[0];
  const bool vec = p.N % 4 == 0 && (!g.bias || aligned16(g.bias)) && (!g.C || (aligned16(g.C) && p.ldc % 4 == 0)) &&
                   (!g.R || (aligned16(g.R) && p.ldr % 4 == 0)) &&
                   (!g.C_lp || (aligned8(g.C_lp) && p.ldc_lp % 4 == 0));
  if (p.row.active()) {
    B2E_CHECK(gemm_tc_row_eligible(p) && vec, kErrInternal, "gemm_tc: row epilogue needs N <= 256 and aligned rows");
    launch_tc<256>(p, vec, s);
  } else {
    launch_tc<128>(p, vec, s);
  }
}

}  // namespace b2e
