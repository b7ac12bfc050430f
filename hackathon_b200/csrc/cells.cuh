// The three state-streaming recurrent steps (the hot loops of the ensemble).
//
// Each reads a row's big state once and writes it once, with the update and the
// contraction against a query vector done in registers in between, exactly the
// contract of the reference's fused Triton steps (model/kernels.py:1-34):
//
//   outer_rows  S[h,k] <- f*S[h,k] + (i*kv[h])*v[k];  out[k] = sum_h q[h]*S_new[h,k]
//               mLSTM (model/kernels.py:143-151, f,i per row/head) and RetNet
//               (model/kernels.py:154-160, f = decay per head, i = 1).
//   ssm_cols    H[p,c] <- decay*H[p,c] + (dt*b[c])*x[p];  y[p] = sum_c c[c]*H_new[p,c]
//               Mamba2 (model/kernels.py:163-171).
//
// Rows are addressed through an optional slot table (row r lives at state +
// slots[r]*row_stride: the engine's per-symbol state table) and an optional mask
// (the reference API: an idle row's state is neither read nor written and its
// output is zero). Live rows come from a device counter or a host constant.
#pragma once
#include "common.cuh"

namespace b2e {

struct RowAddr {
  float* state = nullptr;
  long long row_stride = 0;     // floats between consecutive slots
  const int* slots = nullptr;   // row -> slot; null = identity
  const uint8_t* mask = nullptr;  // null = every row active
  int n_host = 0;
  const int* n_dev = nullptr;
};

struct OuterRowsParams {
  RowAddr at;
  int nh = 0, sh = 0, sk = 0;
  const float* f = nullptr; int f_rs = 0, f_hs = 0;  // factor on the old state
  const float* i = nullptr; int i_rs = 0, i_hs = 0;  // factor on the outer product (null = 1)
  const float* kv = nullptr; int k_rs = 0;           // [row][nh*sh]
  const float* v = nullptr; int v_rs = 0;            // [row][nh*sk]
  const float* q = nullptr; int q_rs = 0;            // [row][nh*sh]
  float* out = nullptr; int o_rs = 0;                // [row][nh*sk]
  int* err = nullptr;                                // device error word for the bulk path's bounded waits, or null
};

struct SsmColsParams {
  RowAddr at;
  int nh = 0, sh = 0, sc = 0;                    // state (nh, sh, sc) per row
  const float* x = nullptr; int x_rs = 0;        // [row][nh*sh]
  const float* b = nullptr; int b_rs = 0;        // [row][sc]
  const float* c = nullptr; int c_rs = 0;        // [row][sc]
  const float* dt = nullptr; int dt_rs = 0;      // [row][nh]
  const float* decay = nullptr; int dc_rs = 0;   // [row][nh]
  float* out = nullptr; int o_rs = 0;            // [row][nh*sh]
  int* err = nullptr;                            // as in OuterRowsParams
};

// Both dispatch to the bulk-copy streaming kernels (stream.cuh) when the
// operands allow, else to the register-streaming kernels here.
void outer_rows(const OuterRowsParams& p, int rows_max, cudaStream_t s, const LaunchCfg& ln = {});
void ssm_cols(const SsmColsParams& p, int rows_max, cudaStream_t s, const LaunchCfg& ln = {});

}  // namespace b2e
