// Shared definitions of the chunked-forward kernels (1) and (2).
#pragma once

#include "common.cuh"

namespace gdn2 {

constexpr int CP = 64;  // padded rows of one chunk (chunk_size <= 64 per pass)
constexpr int KS = 64;  // key-channel slice of the CUDA-core intra kernel

struct ChunkParams {
  int B, T, HV, K, V;
  int C;    // tokens per chunk actually used (min(chunk_size, 64))
  int NC;   // chunks per sequence
  int rep;  // value heads per q/k/g/b view head
  int fuse_epilogue;
  float scale, eps;
  DView q, k, v, g, b, w, gate, out;
  const float* onw;
  float* state;
  // workspace
  float *ws_aqk, *ws_w, *ws_u, *ws_qg, *ws_kd, *ws_gl, *ws_o;
};

// Workspace layout, in floats.
struct ChunkWorkspace {
  size_t aqk, w, u, qg, kd, gl, o, total;
};

inline ChunkWorkspace chunk_workspace_layout(int B, int HV, int T, int K, int V, int C) {
  const size_t nch = (size_t)B * HV * ((T + C - 1) / C);
  ChunkWorkspace L;
  size_t off = 0;
  auto take = [&](size_t n) {
    size_t at = off;
    off += (n + 63) / 64 * 64;  // 256-byte aligned sub-buffers
    return at;
  };
  L.aqk = take(nch * CP * CP);
  L.w = take(nch * CP * K);
  L.u = take(nch * CP * V);
  L.qg = take(nch * CP * K);
  L.kd = take(nch * CP * K);
  L.gl = take(nch * K);
  L.o = take((size_t)B * HV * T * V);
  L.total = off;
  return L;
}

int launch_intra_simt(const ChunkParams& p, int dtype, cudaStream_t st);
int launch_inter_simt(const ChunkParams& p, cudaStream_t st);
int launch_chunk_out(const ChunkParams& p, int dtype, cudaStream_t st);

}  // namespace gdn2
