#pragma once

#include <stdint.h>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "rope_kv.cuh"

namespace omni {

// Decode GEMM (wgemm.cu): y = epilogue(x . w^T) for at most 64 token rows, bf16 in, fp32 accumulate, bf16 out.
enum GemmMode : int {
  kGemmStore = 0,     // y[m, n] = acc
  kGemmResidual = 1,  // y[m, n] = residual[m, n] + acc                       (torch.addmm(residual, x, w.t()))
  kGemmSwiglu = 2,    // w = [gate (n rows); inner (n rows)]: y[m, f] = inner * silu(gate), each rounded to bf16 first
  kGemmRope = 3,      // the QKV product, then RoPE + KV-cache append as rope_kv does it (no qkv is stored): rope.*
};

struct GemmArgs {
  int rows, n, k;  // token rows, output columns, reduction length
  int mode;
  const __nv_bfloat16* residual;
  int64_t ld_res;
  __nv_bfloat16* y;
  int64_t ld_y;
  float* part;    // [grid, 2, NT / 4, 128, 4] fp32 partials of weight tiles split between CTAs
  int* counters;  // [tiles] arrivals on split tiles: zero before and after a call
  int tiles, chunks, grid;
  int cluster;  // 1: stream-K; S > 1: a cluster of S CTAs per tile, reduced through distributed shared memory
  int64_t per;  // (tile, chunk) units per CTA
  int* status;
  RopeArgs rope;  // kGemmRope: positions, cos/sin table, q output, caches (rope.qkv unused)
  int head_dim;   // kGemmRope: n = 3 * rope.heads * head_dim
};

constexpr int kGemmMaxRows = 64;
constexpr int kGemmMaxTiles = 8192;  // weight tiles of one call (n up to 8192 * 128 rows; SwiGLU 8192 * 64)

// Token-tile width (the MMA's N) for `rows` token rows: 16, 32, 48 or 64.
int gemm_token_tile(int rows);
int gemm_tiles(int n, int mode);
// Workspace: per-tile arrival counters (the first gemm_counter_bytes(), the same for every shape; zero on entry and
// zero again after a call that completed) then the partial tiles.
size_t gemm_counter_bytes(int n, int mode);
size_t gemm_workspace_bytes(int rows, int n, int k, int mode);
cudaError_t launch_decode_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, GemmArgs a, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream);

}  // namespace omni
