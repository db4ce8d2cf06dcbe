// tcgen05 GEMM: C[M, N] (bf16) = A[M, K] (bf16, K-major) x B[N, K]^T (bf16, K-major),
// fp32 accumulation in tensor memory.
//
// One CTA (4 warps) owns one 128 x 256 output tile:
//   warp 0 lane 0 : TMA producer -- 4-stage ring of {A 128x64, B 256x64} tiles, 128-byte
//                   swizzle, completion on per-stage "full" mbarriers (no multicast)
//   warp 1 lane 0 : MMA issuer   -- tcgen05.mma.cta_group::1.kind::f16 M=128 N=256 K=16,
//                   four per stage; tcgen05.commit frees the stage ("empty" barrier) and
//                   finally signals "accumulator ready"
//   warp 2        : allocates / frees the 256 TMEM columns of the fp32 accumulator
//   warps 0-3     : epilogue -- tcgen05.ld of their 32 TMEM lanes (= tile rows),
//                   optional fp32 scale and residual add, bf16 store
// A, B and C are plain global memory of this GPU. The optional "gate" lets a
// producer wait, tile by tile, for rows that another agent (a copy engine pulling
// a peer's shard) is still writing: before loading A rows [m0, m0+128) the producer
// waits (bounded) until gate[m0 / gate_rows] >= gate_target.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace axr {

constexpr int GBM = 128, GBN = 256, GBK = 64, GSTAGES = 4;
constexpr int GA_BYTES = GBM * GBK * 2;   // 16 KB
constexpr int GB_BYTES = GBN * GBK * 2;   // 32 KB
constexpr int GSMEM = 1024 + GSTAGES * (GA_BYTES + GB_BYTES) + 256;

struct GemmArgs {
  __nv_bfloat16* c;
  long long ldc;
  const __nv_bfloat16* residual;  // optional [M, N] added in the epilogue
  long long ldr;
  float alpha;
  int M, N, K;
  volatile int* err;
  const volatile int* gate;       // optional per-row-block readiness counters
  int gate_rows;
  int gate_target;
};

__global__ void __launch_bounds__(128, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmB, GemmArgs g) {
  extern __shared__ __align__(1024) char gsm_raw[];
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(gsm_raw) + 1023) & ~uintptr_t(1023));
  char* sA = base;
  char* sB = base + GSTAGES * GA_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + GSTAGES * GB_BYTES);
  uint64_t* empty = full + GSTAGES;
  uint64_t* acc_ready = empty + GSTAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_ready + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * GBN, m0 = blockIdx.y * GBM;
  const int num_k = (g.K + GBK - 1) / GBK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < GSTAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(acc_ready, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  if (warp == 2) {
    tc::tmem_alloc(tmem_slot, GBN);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- producer
    bool ok = true;
    if (g.gate != nullptr) {  // rows of this tile may still be arriving from a peer
      const int blk = m0 / g.gate_rows;
      const unsigned long long t0 = tc::globaltimer();
      while (g.gate[blk] < g.gate_target) {
        if (*g.err != 0 || tc::globaltimer() - t0 > tc::kWaitLimitNs) {
          atomicCAS(const_cast<int*>(g.err), 0, 4);
          ok = false;
          break;
        }
      }
      __threadfence();
    }
    int issued = 0;
    for (int kt = 0; ok && kt < num_k; ++kt) {
      const int s = kt % GSTAGES;
      if (kt >= GSTAGES && !tc::mbar_wait(&empty[s], ((kt / GSTAGES) + 1) & 1, g.err, 1)) { ok = false; break; }
      tc::mbar_arrive_expect_tx(&full[s], GA_BYTES + GB_BYTES);
      tc::tma_load_2d(sA + s * GA_BYTES, &tmA, kt * GBK, m0, &full[s]);
      tc::tma_load_2d(sB + s * GB_BYTES, &tmB, kt * GBK, n0, &full[s]);
      issued = kt + 1;
    }
    if (!ok) {
      // let the loads this thread issued land before the CTA can exit
      for (int kt = max(0, issued - GSTAGES); kt < issued; ++kt)
        tc::mbar_wait_quiet(&full[kt % GSTAGES], (kt / GSTAGES) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = tc::idesc_bf16_f32(GBM, GBN);
    bool ok = true;
    for (int kt = 0; kt < num_k; ++kt) {
      const int s = kt % GSTAGES;
      if (!tc::mbar_wait(&full[s], (kt / GSTAGES) & 1, g.err, 2)) { ok = false; break; }
      tc::tc_fence_after();
      const uint32_t a_addr = tc::smem_u32(sA + s * GA_BYTES);
      const uint32_t b_addr = tc::smem_u32(sB + s * GB_BYTES);
#pragma unroll
      for (int kk = 0; kk < GBK / 16; ++kk) {
        tc::mma_f16_ss(tmem, tc::smem_desc_k_sw128(a_addr + kk * 32), tc::smem_desc_k_sw128(b_addr + kk * 32), idesc,
                       (kt | kk) != 0);
      }
      tc::mma_commit(&empty[s]);
    }
    tc::mma_commit(acc_ready);  // arrives once every MMA above has completed
    if (!ok) tc::mbar_wait_quiet(acc_ready, 0);  // the epilogue may have given up: drain before TMEM is freed
  }
  __syncwarp();

  // ---------------- epilogue (all 4 warps)
  bool ready = tc::mbar_wait(acc_ready, 0, g.err, 3);
  ready = __all_sync(0xffffffffu, ready) && __shfl_sync(0xffffffffu, *g.err, 0) == 0;  // warp-uniform
  tc::tc_fence_after();
  const int row = m0 + warp * 32 + lane;
  if (ready) {
#pragma unroll 1
    for (int c = 0; c < GBN / 16; ++c) {
      uint32_t r[16];
      tc::tmem_ld16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c * 16, r);
      tc::tmem_ld_wait();
      const int col = n0 + c * 16;
      if (row < g.M && col < g.N) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]) * g.alpha;
        if (g.residual != nullptr) {
          const __nv_bfloat16* rp = g.residual + (long long)row * g.ldr + col;
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += (col + j < g.N) ? __bfloat162float(rp[j]) : 0.f;
        }
        __nv_bfloat16* cp = g.c + (long long)row * g.ldc + col;
        if (col + 16 <= g.N && (g.ldc % 8) == 0) {
          uint4 o0 = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                                pack_bf16x2(v[6], v[7]));
          uint4 o1 = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                                pack_bf16x2(v[14], v[15]));
          reinterpret_cast<uint4*>(cp)[0] = o0;
          reinterpret_cast<uint4*>(cp)[1] = o1;
        } else {
          for (int j = 0; j < 16 && col + j < g.N; ++j) cp[j] = __float2bfloat16(v[j]);
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 2) tc::tmem_dealloc(tmem, GBN);
}

// ------------------------------------------------------------------------------- host
namespace {
void make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {GBK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult rc = cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                                             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(rc == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(rc));
}
}  // namespace

void launch_gemm_tc(const void* a, int64_t lda, const void* b, int64_t ldb, void* c, int64_t ldc, const void* residual,
                    int64_t ldr, float alpha, int M, int N, int K, int* err, const int* gate, int gate_rows,
                    int gate_target, cudaStream_t st) {
  CUtensorMap ta, tb;
  make_map(&ta, a, M, K, lda, GBM);
  make_map(&tb, b, N, K, ldb, GBN);
  GemmArgs g{reinterpret_cast<__nv_bfloat16*>(c), ldc, reinterpret_cast<const __nv_bfloat16*>(residual), ldr, alpha,
             M, N, K, err, gate, gate_rows, gate_target};
  static bool attr = false;
  if (!attr) {
    AXR_CHECK_CUDA(cudaFuncSetAttribute(gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GSMEM));
    attr = true;
  }
  dim3 grid((N + GBN - 1) / GBN, (M + GBM - 1) / GBM);
  gemm_tc_kernel<<<grid, 128, GSMEM, st>>>(ta, tb, g);
  AXR_CHECK_CUDA(cudaGetLastError());
}

// a [M, K], b [N, K] (weights in "out x in" order), out [M, N]; err: int32 CUDA tensor
// (>= 1 element) that the kernel sets to a non-zero code if a bounded wait expired.
void gemm_tc(torch::Tensor a, torch::Tensor b, torch::Tensor out, c10::optional<torch::Tensor> residual, double alpha,
             torch::Tensor err) {
  TORCH_CHECK(a.is_cuda() && b.is_cuda() && out.is_cuda(), "gemm_tc: CUDA tensors");
  TORCH_CHECK(a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16 &&
                  out.scalar_type() == torch::kBFloat16,
              "gemm_tc: bf16 operands");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1,
              "gemm_tc: row-major 2D operands");
  TORCH_CHECK(a.size(1) == b.size(1), "gemm_tc: K mismatch");
  TORCH_CHECK(a.size(1) % 8 == 0, "gemm_tc: K must be a multiple of 8");
  TORCH_CHECK(err.scalar_type() == torch::kInt32 && err.is_cuda(), "gemm_tc: err must be an int32 CUDA tensor");
  const int M = a.size(0), N = b.size(0), K = a.size(1);
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm_tc: out shape");
  if (M == 0 || N == 0) return;
  const void* res = nullptr;
  int64_t ldr = 0;
  if (residual.has_value()) {
    TORCH_CHECK(residual->scalar_type() == torch::kBFloat16 && residual->stride(1) == 1, "residual bf16 row-major");
    res = residual->data_ptr();
    ldr = residual->stride(0);
  }
  launch_gemm_tc(a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0), out.data_ptr(), out.stride(0), res, ldr,
                 static_cast<float>(alpha), M, N, K, err.data_ptr<int>(), nullptr, 1, 0,
                 at::cuda::getCurrentCUDAStream());
}

}  // namespace axr
