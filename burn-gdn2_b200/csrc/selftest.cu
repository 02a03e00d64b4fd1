// Diagnostic: one tcgen05 MMA tile per launch in each operand layout the
// chunk kernels use, so the descriptor encodings and TMEM layouts can be
// checked against a host matmul (gdn2_selftest_umma).
#include "common.cuh"
#include "umma.cuh"

namespace gdn2 {

struct SelftestCase {
  int M, N, K;
  bool a_mn, b_mn;
};

__constant__ SelftestCase c_cases[4] = {
    {128, 64, 128, false, true},   // [W; Qg] . S     (A K-major, B MN-major)
    {64, 32, 128, false, false},   // Ks . X^T        (both K-major, M = 64)
    {128, 64, 64, true, true},     // Kd^T . v_new    (A MN-major, B MN-major)
    {128, 128, 64, false, true},   // two N groups    (LBO of the MN-major B)
};

__global__ void __launch_bounds__(128) k_selftest_umma(int test, const float* __restrict__ A,
                                                        const float* __restrict__ B, float* __restrict__ D) {
  extern __shared__ __align__(1024) unsigned char smraw[];
  // SW128 tiles need 1024-byte aligned starts: align the window by hand
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  const SelftestCase tc = c_cases[test];
  unsigned char* sA = sm;               // up to 32 KB
  unsigned char* sB = sm + 32768;       // up to 32 KB
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + 65536);
  uint32_t* tbase = reinterpret_cast<uint32_t*>(sm + 65536 + 8);
  const int tid = threadIdx.x, warp = tid >> 5;

  if (warp == 0) {
    umma::tmem_alloc(tbase, 128);
    umma::tmem_relinquish();
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  // A logical [M][K], B logical [K][N], both row-major f32 in global memory
  for (int i = tid; i < tc.M * tc.K; i += 128) {
    const int m = i / tc.K, k = i % tc.K;
    const uint32_t off = tc.a_mn ? umma::mnmaj_off(k, m, tc.K) : umma::kmaj_off(m, k, tc.M);
    *reinterpret_cast<__nv_bfloat16*>(sA + off) = __float2bfloat16_rn(A[i]);
  }
  for (int i = tid; i < tc.K * tc.N; i += 128) {
    const int k = i / tc.N, n = i % tc.N;
    const uint32_t off = tc.b_mn ? umma::mnmaj_off(k, n, tc.K) : umma::kmaj_off(n, k, tc.N);
    *reinterpret_cast<__nv_bfloat16*>(sB + off) = __float2bfloat16_rn(B[i]);
  }
  fence_proxy_async_smem();
  umma::fence_before_sync();
  __syncthreads();
  umma::fence_after_sync();
  const uint32_t t0 = *tbase;
  if (tid == 0) {
    const uint32_t idesc = umma::idesc_bf16(tc.M, tc.N, tc.a_mn, tc.b_mn);
    const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
    for (int j = 0; j < tc.K / 16; ++j) {
      const uint64_t ad = tc.a_mn ? umma::desc_mnmaj(a0, tc.K, j) : umma::desc_kmaj(a0, tc.M, j);
      const uint64_t bd = tc.b_mn ? umma::desc_mnmaj(b0, tc.K, j) : umma::desc_kmaj(b0, tc.N, j);
      umma::mma_bf16(t0, ad, bd, idesc, j > 0);
    }
    umma::commit(bar);
  }
  mbar_wait_bounded(bar, 0);
  umma::fence_after_sync();
  // M = 128: row = TMEM lane.  M = 64: row r lives in lane (r % 16) + 32 (r / 16).
  const int lane_row = tid;  // lane of this thread inside the warp's sub-partition
  int row = -1;
  if (tc.M == 128) row = lane_row;
  else if ((tid & 31) < 16) row = (tid >> 5) * 16 + (tid & 31);
  for (int c0 = 0; c0 < tc.N; c0 += 16) {
    float v[16];
    umma::ld16(umma::taddr(t0, warp * 32, c0), v);
    umma::wait_ld();
    if (row >= 0)
      for (int j = 0; j < 16; ++j) D[row * tc.N + c0 + j] = v[j];
  }
  umma::fence_before_sync();
  __syncthreads();
  if (warp == 0) umma::tmem_dealloc(t0, 128);
}

int selftest_umma(int test, const float* A, const float* B, float* D, cudaStream_t st) {
  const size_t smem = 65536 + 64 + 1024;
  cudaError_t e = cudaFuncSetAttribute((const void*)k_selftest_umma, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return check_cuda(e, "selftest smem");
  k_selftest_umma<<<1, 128, smem, st>>>(test, A, B, D);
  return check_cuda(cudaGetLastError(), "selftest launch");
}

// Diagnostic of the failure path every kernel's waits share: thread 0 waits
// on an mbarrier through mbar_wait_bounded with a limit of `spins` rounds.
// With arrive = 0 nothing ever arrives, so the wait gives up, records
// DEVERR_MBAR_TIMEOUT and the kernel returns normally (no trap, the context
// stays usable); with arrive = 1 the phase completes at once.
static __device__ int g_wait_completed = -1;

__global__ void k_selftest_wait(unsigned spins, int arrive) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (arrive) mbar_arrive(&bar);
    g_wait_completed = mbar_wait_bounded(&bar, 0, spins) ? 1 : 0;
  }
}

int selftest_wait(unsigned spins, int arrive, int* completed) {
  k_selftest_wait<<<1, 32>>>(spins, arrive);
  int rc = check_cuda(cudaGetLastError(), "selftest wait launch");
  if (rc) return rc;
  rc = check_cuda(cudaDeviceSynchronize(), "selftest wait");
  if (rc) return rc;
  return check_cuda(cudaMemcpyFromSymbol(completed, g_wait_completed, sizeof(int)), "selftest wait result");
}

GDN2_DEVICE_ERROR_READER(read_device_errors_selftest)

}  // namespace gdn2
