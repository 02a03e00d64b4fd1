// Tensor-core (tcgen05) chunk path: shared definitions of the chunk-intra
// and chunk-inter kernels for bf16 inputs, K = 128 key channels, chunk 64.
//
// The intra kernel writes, per (b, hv, chunk), one record whose matrix
// parts are byte images of the inter kernel's shared-memory operand tiles
// (128-byte-swizzled canonical layouts, see umma.cuh), so the inter kernel
// moves each part with a single bulk copy:
//   WQ  [128][128] K-major : rows 0..63 W = (I+Akk)^-1 (b k gamma),
//                            rows 64..127 Qg = scale q gamma
//   AQK [64][64]   K-major : scale * causal(q k^T decay)       (forward.rs:159-187)
//   KD  [64][128]  MN-major: k exp(G_last - G)  (A operand of Kd^T v_new)
//   U   [VS][64][VT] bf16 row-major per column slice: (I+Akk)^-1 (w v);
//                            16-byte chunk j of row r sits at chunk j ^ (r & 7),
//                            so the inter kernel's per-lane row reads are free
//                            of shared-memory bank conflicts
//   GL  [128] f32          : gamma_last = exp(G_last)
#pragma once

#include "chunk.cuh"

namespace gdn2 {

constexpr int TC_K = 128;
constexpr int TC_C = 64;

struct TcRecord {
  size_t wq, aqk, kd, u, gl, bytes;
};

__host__ __device__ inline TcRecord tc_record_layout(int V) {
  TcRecord r;
  r.wq = 0;
  r.aqk = r.wq + 128 * 128 * 2;
  r.kd = r.aqk + 64 * 64 * 2;
  r.u = r.kd + 64 * 128 * 2;
  r.gl = r.u + (size_t)64 * V * 2;
  r.bytes = (r.gl + TC_K * 4 + 1023) / 1024 * 1024;
  return r;
}

struct TcParams {
  int B, T, HV, V, NC, rep, vt, vsplit;
  float scale, eps;
  int fuse_epilogue;
  DView q, k, v, g, b, w, gate, out;
  const float* onw;
  float* state;
  unsigned char* rec;  // NC records per (b, hv), record bytes each
  size_t rec_bytes;
  unsigned char* scratch;  // split-operand intra kernel: one L2-resident slot per CTA (after the records)
  // chunk-parallel state scan of the split-operand inter kernel (nseg = 1: one CTA walks the whole chain):
  // the chain's chunks in nseg segments of seg_len; phase A computes each segment's end state from zero and
  // its state transition, then (nseg > 1) the segments run from their start states.
  int nseg, seg_len;
  float* seg_state;  // [B][HV][nseg][K][V]: slot s = the start state of segment s
  float* seg_trans;  // [B][HV][nseg - 1][K][K]: the transition over segment s
};

int launch_intra_tc(const TcParams& p, cudaStream_t st);
int launch_inter_tc(const TcParams& p, cudaStream_t st);
bool tc_supported(int K, int V, int C, int dtype);

}  // namespace gdn2
