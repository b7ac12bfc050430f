// tcgen05 (5th-generation tensor core) GEMM for the CastLinear projections.
//
// C[m, n] = epilogue( sum_k A[m, k] * W[n, k] ), A and W both bf16 (or both f16)
// in global memory, f32 accumulation in tensor memory. The projections here are
// skinny (a few thousand rows, N and K of a few hundred), so the tensor core
// computes the transposed tile: its 128-wide M side runs over output features
// (W rows) and its N side over BR activation rows. One CTA owns BR rows x NT*128
// features, so a tile of whole rows (N <= 256) needs only BR = 32 rows and a
// step of 4096 rows still spreads over 128 CTAs.
//   warp 0     one thread issues TMA loads of the W tile (NT*128 rows x 64 K)
//              and the A tile (BR rows x 64 K), 128-byte swizzle, into a
//              3-stage shared-memory ring;
//   warp 1     allocates NT*BR TMEM columns; one thread issues tcgen05.mma
//              (M=128 features, N=BR rows, K=16 per instruction) per 128-feature
//              half and commits each stage back to the producer and the finished
//              accumulator to the epilogue;
//   warps 2-9  epilogue (kEpiWarps = 8), in two phases. Phase 1: each warp
//              reads its 32-lane TMEM quadrant (warps w and w+4 share one quadrant
//              and split its 32-row chunks; one thread per feature, 32 rows per
//              tcgen05.ld),
//              applies bias, CastLinear rounding and activation, and stages the
//              tile row-major in the now idle operand ring. Phase 2: each warp
//              takes whole rows (lane = 16-byte column unit) and writes them with
//              row-contiguous stores, adding the residual; optional row work
//              (RowEpi: LayerNorm, a second residual, the next RMSNorm, a dot
//              product) runs here with warp-shuffle reductions.
// Every mbarrier wait is bounded: past ~1 s the kernel records an error code,
// stops issuing work, waits (bounded) for what it issued, frees its TMEM and
// returns. TMA loads here never use cluster multicast.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "gemm.cuh"
#include "mbarrier.cuh"
#include "stream.cuh"

namespace b2e {
namespace {

constexpr int FT = 128, BK = 64;  // FT: features per MMA (its M)
constexpr int kEpiWarps = 8, kEpiThreads = 32 * kEpiWarps;
constexpr int THREADS = 64 + kEpiThreads;  // producer warp, MMA warp, epilogue warps
constexpr int kMaxStages = 8;                    // ring depth is chosen per launch
constexpr size_t kSmemBarriers = 1024 + 256;     // 1024-byte alignment slack + barriers

template <int NT, int BR>
struct Cfg {
  static constexpr int NOUT = NT * FT;                   // features per CTA
  static constexpr uint32_t TILE_W = NOUT * BK * 2;      // NT x 16 KB
  static constexpr uint32_t TILE_X = BR * BK * 2;        // BR x 128 B
  static constexpr uint32_t STAGE = TILE_W + TILE_X;     // multiple of 1024 (swizzle atoms)
  static constexpr uint32_t TMEM_COLS = NT * BR;         // power of two >= 32
  // the epilogue stages BR x NOUT floats in the ring
  static constexpr int MIN_STAGES = (BR * NOUT * 4 + STAGE - 1) / STAGE > 2 ? (BR * NOUT * 4 + STAGE - 1) / STAGE : 2;
  static_assert(STAGE % 1024 == 0, "stage bases must stay 1024-byte aligned");
  static_assert(TMEM_COLS >= 32 && (TMEM_COLS & (TMEM_COLS - 1)) == 0, "TMEM allocation is a power of two >= 32");
  static_assert(MIN_STAGES <= kMaxStages, "epilogue stage must fit the ring");
  static size_t smem(int stages) { return size_t(stages) * STAGE + kSmemBarriers; }
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
  int stages;  // ring depth, MIN_STAGES..kMaxStages
};

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

// Instruction descriptor, kind::f16: f32 accumulator, A/B type, both K-major,
// M = FT (128) features, N = n rows.
__host__ __device__ constexpr uint32_t instr_desc(int lp, int n) {
  const uint32_t ab = lp == kBF16 ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(FT >> 4) << 24);
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


// Row work of the epilogue, fixed per instantiation so that each loop carries
// only the instructions it needs (the epilogue is issue-latency bound: one or
// two warps per SM sub-partition work through dependent chains).
enum RowMode : int {
  kRowPlain = 0,  // C / C_lp (+ R)
  kRowNorm = 1,   // + RMSNorm -> T / T_lp
  kRowLnNorm = 2, // + LayerNorm, + R2, then RMSNorm -> T / T_lp
  kRowDot = 3,    // + dot product -> dot_out
};

int row_mode(const RowEpi& r) {
  if (r.dot_w) return kRowDot;
  if (r.ln_w) return kRowLnNorm;
  if (r.norm_w) return kRowNorm;
  return kRowPlain;
}

template <int NT, int BR, int MODE>
__global__ void __launch_bounds__(THREADS)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, const TcEpi e) {
  using K = Cfg<NT, BR>;
  constexpr int NOUT = K::NOUT;
  constexpr int UPR = NOUT / 4;  // 16-byte units per tile row
  constexpr int UPL = UPR / 32;  // units per lane in phase 2
  const int m0 = blockIdx.y * BR, n0 = blockIdx.x * NOUT;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base by pointer arithmetic on the shared array, so the
  // compiler keeps shared-space accesses (no generic loads and stores that it
  // must order against the global stores of the epilogue)
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int S = e.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(S) * K::STAGE);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  // Set-up that touches no global data: it overlaps the previous kernel's tail.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tw)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tx)) : "memory");
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
  // TMEM is held from here on; the successor may start only after this point.
  pdl_wait();
  const int M = live_rows(e.M_dev, e.M_max);
  const bool live = m0 < M;  // uniform over the CTA
  const int nkb = (e.K + BK - 1) / BK;

  if (!live) {
    // no rows: nothing issued, nothing to wait for
  } else if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer
      int issued = 0;
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (kb >= S && !mbar_wait(&empty[s], ph ^ 1, abort_flag)) {
          if (!*abort_flag) atomicExch(e.err, kTcTimeoutProducer);
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * K::STAGE;
        mbar_expect_tx(&full[s], K::STAGE);
        tma_load_2d(st, &tw, kb * BK, n0, &full[s]);
        tma_load_2d(st + K::TILE_W, &tx, kb * BK, m0, &full[s]);
        ++issued;
      }
      if (*abort_flag) {
        // drain: every load issued lands before the CTA leaves (bounded)
        volatile int never = 0;
        for (int kb = max(0, issued - S); kb < issued; ++kb)
          mbar_wait(&full[kb % S], (kb / S) & 1, &never);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer: D_h[f, r] += W[h*128 + f, k] * A[r, k]
      const uint32_t idesc = instr_desc(e.lp, BR);
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % S;
        const uint32_t ph = (kb / S) & 1;
        if (!mbar_wait(&full[s], ph, abort_flag)) {
          if (!*abort_flag) atomicExch(e.err, kTcTimeoutMma);
          *abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t w0 = smem_u32(smem + s * K::STAGE), x0 = w0 + K::TILE_W;
#pragma unroll
        for (int h = 0; h < NT; ++h)
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)  // K=16 per instruction: +32 bytes inside the swizzled row
            mma_f16(tmem + uint32_t(h * BR), smem_desc(w0 + h * FT * 128 + k * 32), smem_desc(x0 + k * 32), idesc,
                    (kb | k) != 0);
        mma_commit(&empty[s]);  // frees the stage once these MMAs have read it
      }
      mma_commit(done);  // accumulator complete (covers every MMA issued)
    }
  } else {
    // ---- epilogue: warps 2..9. TMEM lane quadrant q = warp % 4 (features
    // q*32..q*32+31); the two warps of a quadrant split its 32-row chunks.
    // While the main loop runs, load what the row pass needs besides the
    // accumulator: this warp's first kPre rows of R (and R2), and the column
    // weights of the row work.
    constexpr int kPre = 4;
    const int rows = min(BR, M - m0);
    float4 pre_r[kPre][UPL], pre_r2[kPre][UPL], w_a[UPL], w_b[UPL];
    if (e.vec) {
      const float* R = e.R;
      const float* R2 = MODE == kRowLnNorm ? e.row.R2 : nullptr;
#pragma unroll
      for (int u = 0; u < UPL; ++u) {
        const int n = n0 + (lane + 32 * u) * 4;
        const bool in = n < e.N;
#pragma unroll
        for (int b = 0; b < kPre; ++b) {
          const int r = warp - 2 + kEpiWarps * b;
          const bool ok_r = in && r < rows;
          pre_r[b][u] = (ok_r && R) ? *reinterpret_cast<const float4*>(R + size_t(m0 + r) * e.ldr + n)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
          pre_r2[b][u] = (ok_r && R2) ? *reinterpret_cast<const float4*>(R2 + size_t(m0 + r) * e.row.ldr2 + n)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        const float* wa = MODE == kRowLnNorm ? e.row.ln_w : MODE == kRowNorm ? e.row.norm_w : MODE == kRowDot ? e.row.dot_w : nullptr;
        const float* wb = MODE == kRowLnNorm ? e.row.norm_w : nullptr;
        w_a[u] = (in && wa) ? *reinterpret_cast<const float4*>(wa + n) : make_float4(0.f, 0.f, 0.f, 0.f);
        w_b[u] = (in && wb) ? *reinterpret_cast<const float4*>(wb + n) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    volatile int never = 0;  // the MMA thread always commits `done`, even after an abort
    const bool ok = mbar_wait(done, 0, &never);
    if (!ok) {
      atomicExch(e.err, kTcTimeoutEpilogue);
      *abort_flag = 1;
    }
    // Both named barriers below are reached by all eight epilogue warps whatever
    // happens, so an error path cannot leave a warp waiting; `go` is read once.
    asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
    const bool go = ok && !*abort_flag;
    const int q = warp & 3, half = (warp - 2) >> 2;
    if (go) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    // Phase 1: per feature (this thread's TMEM lane) bias, rounding, activation;
    // the tile goes to shared memory row-major (BR x NOUT floats; the operand
    // ring is idle once `done` fired). For a fixed row the 32 lanes write 32
    // consecutive floats: no bank conflicts.
    float* stage = reinterpret_cast<float*>(smem);
    constexpr int CH = BR / 32;  // 32-row chunks per 128-feature half
#pragma unroll 1
    for (int k = half; k < NT * CH; k += 2) {
      const int h = k / CH, c = (k % CH) * 32;
      const int fb = h * FT + q * 32;
      if (!go || n0 + fb >= e.N) continue;  // warp-uniform
      const int n = n0 + fb + lane;
      const float b = (e.bias && n < e.N) ? load_as(e.bias_type, e.bias, n) : 0.0f;
      float v[32];
      tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(h * BR + c), v);
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 x = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        if (e.bias) x = make_float4(x.x + b, x.y + b, x.z + b, x.w + b);
        if (e.round_out) x = round4_lp(e.lp, x);
        if (e.act == kActRelu) {
          x.x = fmaxf(x.x, 0.f); x.y = fmaxf(x.y, 0.f); x.z = fmaxf(x.z, 0.f); x.w = fmaxf(x.w, 0.f);
        }
        float* col = stage + size_t(c + j) * NOUT + fb + lane;
        col[0] = x.x;
        col[NOUT] = x.y;
        col[2 * NOUT] = x.z;
        col[3 * NOUT] = x.w;
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
    // Phase 2: whole rows per warp (rows warp-2, warp+6, ...); lane l owns
    // 16-byte units l, l+32, ... of a row.
    const float4* stage4 = reinterpret_cast<const float4*>(smem);
    if (go && e.vec) {
      const float* R = e.R;
      float* C = e.C;
      void* C_lp = e.C_lp;
      const int ldr = e.ldr, ldc = e.ldc, ldc_lp = e.ldc_lp, N = e.N, lp = e.lp;
      const float invN = 1.0f / float(N);
      const RowEpi re = e.row;
      // One row: x = staged + R, row work, stores. rr/rr2: R and R2 of the row.
      auto row = [&](int r, const float4 (&rr)[UPL], const float4 (&rr2)[UPL]) {
        const size_t mm = size_t(m0 + r);
        float4 x[UPL];
        bool in[UPL];
#pragma unroll
        for (int u = 0; u < UPL; ++u) {
          const int unit = lane + 32 * u;
          in[u] = n0 + unit * 4 < N;
          x[u] = in[u] ? f4add(stage4[r * UPR + unit], rr[u]) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if constexpr (MODE == kRowLnNorm) {
          // LayerNorm(bias=False): two-pass mean and biased variance, then + R2
          float sm = 0.f;
#pragma unroll
          for (int u = 0; u < UPL; ++u) sm += f4sum(x[u]);
          const float mu = warp_sum(sm) * invN;
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
              const float4 w = w_a[u];
              x[u] = f4add(make_float4((x[u].x - mu) * rs * w.x, (x[u].y - mu) * rs * w.y, (x[u].z - mu) * rs * w.z,
                                       (x[u].w - mu) * rs * w.w), rr2[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < UPL; ++u)
          if (in[u]) {
            const int n = n0 + (lane + 32 * u) * 4;
            if (C) *reinterpret_cast<float4*>(C + mm * ldc + n) = x[u];
            if (C_lp) store4_lp(lp, C_lp, mm * ldc_lp + n, x[u]);
          }
        if constexpr (MODE == kRowNorm || MODE == kRowLnNorm) {  // nn.RMSNorm of the finished row
          float ss = 0.f;
#pragma unroll
          for (int u = 0; u < UPL; ++u)
            ss += f4sum(make_float4(x[u].x * x[u].x, x[u].y * x[u].y, x[u].z * x[u].z, x[u].w * x[u].w));
          const float inv = 1.0f / sqrtf(warp_sum(ss) * invN + re.norm_eps);
#pragma unroll
          for (int u = 0; u < UPL; ++u)
            if (in[u]) {
              const int n = n0 + (lane + 32 * u) * 4;
              const float4 w = MODE == kRowLnNorm ? w_b[u] : w_a[u];
              const float4 t = make_float4(x[u].x * inv * w.x, x[u].y * inv * w.y, x[u].z * inv * w.z, x[u].w * inv * w.w);
              if (re.T) *reinterpret_cast<float4*>(re.T + mm * re.ldt + n) = t;
              if (re.T_lp) store4_lp(lp, re.T_lp, mm * re.ldt + n, t);
            }
        }
        if constexpr (MODE == kRowDot) {  // output_proj: v . w + b
          float d = 0.f;
#pragma unroll
          for (int u = 0; u < UPL; ++u)
            if (in[u]) d += f4sum(make_float4(x[u].x * w_a[u].x, x[u].y * w_a[u].y, x[u].z * w_a[u].z, x[u].w * w_a[u].w));
          d = warp_sum(d);
          if (lane == 0) re.dot_out[mm * re.dot_ld + re.dot_col] = d + re.dot_b[0];
        }
      };
#pragma unroll
      for (int b = 0; b < kPre; ++b) {
        const int r = warp - 2 + kEpiWarps * b;
        if (r < rows) row(r, pre_r[b], pre_r2[b]);
      }
      for (int r = warp - 2 + kEpiWarps * kPre; r < rows; r += kEpiWarps) {
        float4 rr[UPL], rr2[UPL];
#pragma unroll
        for (int u = 0; u < UPL; ++u) {
          const int n = n0 + (lane + 32 * u) * 4;
          const bool in = n < N;
          rr[u] = (in && R) ? *reinterpret_cast<const float4*>(R + size_t(m0 + r) * ldr + n) : make_float4(0.f, 0.f, 0.f, 0.f);
          rr2[u] = (in && MODE == kRowLnNorm && re.R2)
                       ? *reinterpret_cast<const float4*>(re.R2 + size_t(m0 + r) * re.ldr2 + n)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        row(r, rr, rr2);
      }
    } else if (go) {
      // unaligned rows (plain epilogue only: row work needs aligned rows)
      for (int r = warp - 2; r < rows; r += kEpiWarps) {
        const int mm = m0 + r;
        for (int u = 0; u < UPL; ++u)
          for (int i = 0; i < 4; ++i) {
            const int f = (lane + 32 * u) * 4 + i, n = n0 + f;
            if (n >= e.N) continue;
            float x = stage[size_t(r) * NOUT + f];
            if (e.R) x += e.R[size_t(mm) * e.ldr + n];
            if (e.C) e.C[size_t(mm) * e.ldc + n] = x;
            if (e.C_lp) store_as(e.lp, e.C_lp, size_t(mm) * e.ldc_lp + n, x);
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

constexpr size_t kSmemPerSm = 228 * 1024;   // shared memory of one SM
constexpr size_t kSmemPerCta = 227 * 1024;  // largest dynamic allocation of one CTA
constexpr size_t kSmemReserved = 1024;      // the system's share of each resident CTA
// A GEMM CTA stays within what an SM has left beside one bulk state-streaming
// CTA (stream.cuh), so the projections of one tower can run on the same SMs
// while another tower's state streams.
constexpr size_t kSmemGemmCap = kSmemPerSm - (stream_cfg::kStreamSmem + kSmemReserved) - kSmemReserved;

// One candidate tile shape: CTAs, resident CTAs per SM, ring depth, and a cost
// estimate in microseconds: each wave pays a fixed latency (TMA round trips,
// epilogue, launch), and each SM moves its CTAs' operand and output bytes.
struct TilePlan {
  int nt = 0, br = 0, stages = 0;
  double cost = 1e30;
};

template <int NT, int BR>
void plan(const GemmParams& p, TilePlan& best) {
  using K = Cfg<NT, BR>;
  const long ctas = long(ceil_div(p.N, K::NOUT)) * ceil_div(p.M_max, BR);
  const int nkb = ceil_div(p.K, BK);
  const int cap = std::min(kMaxStages, std::max(nkb, K::MIN_STAGES));
  for (int occ = 3; occ >= 1; --occ) {
    const size_t per_cta = std::min(kSmemGemmCap, kSmemPerSm / occ - kSmemReserved);
    if (per_cta < K::smem(K::MIN_STAGES)) continue;
    const int st = std::min<int>(cap, int((per_cta - kSmemBarriers) / K::STAGE));
    if (occ > 1 && ctas <= 148L * (occ - 1)) continue;  // fewer CTAs per SM suffice: keep the deeper ring
    const long waves = (ctas + 148L * occ - 1) / (148L * occ);
    const long per_sm = (ctas + 147) / 148;
    const double bytes = double(nkb) * K::STAGE + double(BR) * K::NOUT * 4;
    const double cost = 3.0 * waves + per_sm * bytes / 150e3;  // 150 GB/s per SM, in us
    if (cost < best.cost) best = {NT, BR, st, cost};
    return;
  }
}

template <int NT, int BR, int MODE>
void launch_tc(const GemmParams& p, bool vec, int stages, cudaStream_t s) {
  using K = Cfg<NT, BR>;
  CUtensorMap tw, tx;
  make_map(&tw, p.g[0].W, p.w_type, uint64_t(p.K), uint64_t(p.N), uint64_t(p.ldw), K::NOUT);
  make_map(&tx, p.g[0].A, p.w_type, uint64_t(p.K), uint64_t(p.M_max), uint64_t(p.lda), BR);
  const GemmGroup& g = p.g[0];
  TcEpi e{g.bias, p.bias_type, g.C, p.ldc, g.C_lp, p.ldc_lp, g.R, p.ldr, p.M_max, p.M_dev,
          p.N, p.K, p.w_type, p.round_out, p.act, p.err, vec ? 1 : 0, p.row, p.row.active() ? 1 : 0, stages};
  dim3 grid(ceil_div(p.N, K::NOUT), ceil_div(p.M_max, BR));
  launch_k(p.ln, gemm_tc_kernel<NT, BR, MODE>, grid, dim3(THREADS), K::smem(stages), s, tw, tx, e);
}

template <int NT, int BR>
void launch_mode(const GemmParams& p, bool vec, int stages, cudaStream_t s) {
  switch (row_mode(p.row)) {
    case kRowNorm: return launch_tc<NT, BR, kRowNorm>(p, vec, stages, s);
    case kRowLnNorm: return launch_tc<NT, BR, kRowLnNorm>(p, vec, stages, s);
    case kRowDot: return launch_tc<NT, BR, kRowDot>(p, vec, stages, s);
    default: return launch_tc<NT, BR, kRowPlain>(p, vec, stages, s);
  }
}

template <int NT>
void launch_nt(const GemmParams& p, bool vec, const TilePlan& t, cudaStream_t s) {
  if (t.br == 128)
    launch_mode<NT, 128>(p, vec, t.stages, s);
  else if (t.br == 64)
    launch_mode<NT, 64>(p, vec, t.stages, s);
  else
    launch_mode<NT, 32>(p, vec, t.stages, s);
}

bool row_buffers_ok(const GemmParams& p) {
  const RowEpi& r = p.row;
  return (!r.ln_w || aligned16(r.ln_w)) && (!r.R2 || (aligned16(r.R2) && r.ldr2 % 4 == 0)) &&
         (!r.norm_w || aligned16(r.norm_w)) && (!r.T || (aligned16(r.T) && r.ldt % 4 == 0)) &&
         (!r.T_lp || (aligned8(r.T_lp) && r.ldt % 4 == 0)) &&
         (!r.dot_w || (aligned16(r.dot_w) && r.dot_b && r.dot_out)) &&
         (!r.ln_w || r.norm_w) && (!r.R2 || r.ln_w);  // LayerNorm (+R2) runs only ahead of an RMSNorm
}

template <int NT, int BR, int MODE>
void set_smem1() {
  using K = Cfg<NT, BR>;
  const size_t mx = std::min(kSmemPerCta, K::smem(kMaxStages));
  B2E_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<NT, BR, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(mx)));
}

template <int NT, int BR>
void set_smem() {
  set_smem1<NT, BR, kRowPlain>();
  set_smem1<NT, BR, kRowNorm>();
  set_smem1<NT, BR, kRowLnNorm>();
  set_smem1<NT, BR, kRowDot>();
}

}  // namespace

void gemm_tc_init() {
  gemm_simt_init();
  set_smem<1, 32>();
  set_smem<1, 64>();
  set_smem<1, 128>();
  set_smem<2, 32>();
  set_smem<2, 64>();
  set_smem<2, 128>();
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
  // A row epilogue needs whole rows in one CTA: 128 features for N <= 128,
  // else 256. Otherwise every shape competes on the cost estimate.
  const bool row = p.row.active();
  if (row) B2E_CHECK(gemm_tc_row_eligible(p) && vec, kErrInternal, "gemm_tc: row epilogue needs N <= 256 and aligned rows");
  TilePlan t;
  if (!row || p.N <= FT) {
    plan<1, 32>(p, t);
    plan<1, 64>(p, t);
    plan<1, 128>(p, t);
  }
  if (!row || p.N > FT) {
    plan<2, 32>(p, t);
    plan<2, 64>(p, t);
    plan<2, 128>(p, t);
  }
  B2E_CHECK(t.nt != 0, kErrInternal, "gemm_tc: no tile shape fits");
  if (t.nt == 2)
    launch_nt<2>(p, vec, t, s);
  else
    launch_nt<1>(p, vec, t, s);
}

}  // namespace b2e
