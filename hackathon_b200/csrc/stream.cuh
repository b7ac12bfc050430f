// HBM-streaming recurrent state steps moved by TMA bulk copies.
//
// Same operands and arithmetic as outer_rows / ssm_cols (cells.cuh), which
// dispatch here whenever the shapes and alignments allow. One persistent CTA per
// SM: one thread streams (row, head group) blocks of state, together with the
// block's operand vectors, global -> shared with cp.async.bulk into a 3-stage
// ring; eight warps update the block in shared memory and contract it; one
// thread writes it back with a bulk store. 288 threads keep ~70 KB of loads in
// flight per SM and leave most of the SM's threads and registers, and half its
// shared memory, to kernels running beside it.
#pragma once
#include "cells.cuh"

namespace b2e {

namespace stream_cfg {
constexpr int kCW = 8;                      // compute warps (and one producer warp)
constexpr int kStages = 3;                  // ring depth
constexpr unsigned kStateMax = 32 * 1024;   // state bytes of one item
constexpr unsigned kOpsMax = 4 * 1024;      // operand bytes of one item
// dynamic shared memory of one CTA: alignment slack, ring, barriers, partials
constexpr size_t kStreamSmem = 128 + size_t(kStages) * (kStateMax + kOpsMax) + 256 + size_t(kCW) * 32 * 16;
}  // namespace stream_cfg

void stream_init();  // per device (idempotent); the engine calls it before any capture
// Waves of the state kernels' grid when a launch leaves it to the process
// (LaunchCfg::bulk_waves < 0): 8 unless set; set returns the previous value.
int state_kernel_waves();
int set_state_kernel_waves(int waves);
bool outer_rows_bulk_ok(const OuterRowsParams& p);
bool ssm_cols_bulk_ok(const SsmColsParams& p);
void outer_rows_bulk(const OuterRowsParams& p, int rows_max, cudaStream_t s, const LaunchCfg& ln);
void ssm_cols_bulk(const SsmColsParams& p, int rows_max, cudaStream_t s, const LaunchCfg& ln);

}  // namespace b2e
