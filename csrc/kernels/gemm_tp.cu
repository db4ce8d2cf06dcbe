// Persistent tcgen05 GEMM with the tensor-parallel collectives fused in.
//
//   out = A x B^T, A [M, K] bf16, B [N, K] bf16 (weights "out x in"), fp32 accumulate.
//
// Modes
//   PLAIN : A is local. (Persistent version of gemm_tc with the epilogue of tile i
//           overlapping the MMAs of tile i+1: two 256-column TMEM accumulators.)
//   AG    : all-gather -> GEMM. A is the row-gather of the world's shards
//           A_p [M/P, K] (one per GPU, in symmetric memory). The CTAs' epilogue warps
//           first pull the peer row blocks this CTA is assigned, 128 rows at a time,
//           with plain 16-byte loads from the peer's memory over NVLink into a local
//           staging buffer, then publish a per-block flag; the TMA producer of any CTA
//           that needs a remote block waits (bounded) for its flag and then loads it from
//           the local staging buffer. Tiles of the local shard are scheduled first, so
//           the MMAs start while the pulls are in flight. Each remote byte crosses
//           NVLink once.
//   RS    : GEMM -> reduce-scatter. Every GPU computes a partial out [M, N] from its
//           K-shard. The epilogue stores each bf16 partial tile straight into the
//           receive slot of the GPU that owns those rows (P2P stores over NVLink) and
//           bumps that GPU's per-row-block arrival counter (system-scope atomic). After
//           its tiles, each GPU reduces its own row blocks as soon as all P x N/256
//           partial tiles of a block have arrived, then takes those arrivals back off
//           the counter (so the next call may use another row count). Counters and
//           receive slots alternate between two parities: a peer may already push
//           partials of call e+1 while this GPU still reduces call e, never of e+2.
// No TMA touches peer memory; no multicast is used. Every wait is bounded (2 s) and
// reports through the error flag instead of hanging; the launch is cooperative, so
// every CTA whose flags another CTA waits on is resident.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "tc_common.cuh"

namespace axr {

constexpr int TBM = 128, TBN = 256, TBK = 64, TST = 4;
constexpr int TA_BYTES = TBM * TBK * 2, TB_BYTES = TBN * TBK * 2;
constexpr int TSMEM = 1024 + TST * (TA_BYTES + TB_BYTES) + 256;
constexpr int MODE_PLAIN = 0, MODE_AG = 1, MODE_RS = 2;

struct TpArgs {
  __nv_bfloat16* c;  // PLAIN/AG output [M, N]
  long long ldc;
  int M, N, K;
  int rank, world, rows_per_rank;  // AG/RS: M = world * rows_per_rank
  int mode;
  int epoch;  // 1, 2, 3, ... per call of this mode on this communicator (same on every GPU)
  // AG
  const int64_t* peer_a;  // [world] base addresses of the peers' A shards [rows_per_rank, K]
  __nv_bfloat16* staging;   // local [M, K]; the TMA map of A covers it
  int* block_flag;          // local [M / 128]: epoch when the block is in staging
  int* ready;               // local [world]: epoch when peer p's shard is ready
  const int64_t* peer_ready;  // [world] addresses of each peer's `ready` array
  // RS
  const int64_t* peer_recv;  // [world] base of each peer's receive area [2][world][rows_per_rank][N]
  const int64_t* peer_cnt;   // [world] base of each peer's arrival counters [rows_per_rank/128][2 parities]
  __nv_bfloat16* recv;         // local receive area
  int* cnt;                    // local counters
  __nv_bfloat16* out_rs;       // [rows_per_rank, N] reduced output of this GPU
  volatile int* err;
};

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(int* p, int v) {
  asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// bounded wait until *p >= target
template <bool SYS>
__device__ __forceinline__ bool wait_geq(const int* p, int target, volatile int* err, int code) {
  const unsigned long long t0 = tc::globaltimer();
  while ((SYS ? ld_acquire_sys(p) : ld_acquire_gpu(p)) < target) {
    if (*err != 0) return false;
    if (tc::globaltimer() - t0 > tc::kWaitLimitNs) {
      atomicCAS(const_cast<int*>(err), 0, code);
      return false;
    }
  }
  return true;
}

__global__ void __launch_bounds__(192, 1) gemm_tp_kernel(const __grid_constant__ CUtensorMap tmA,
                                                         const __grid_constant__ CUtensorMap tmB, TpArgs g) {
  extern __shared__ __align__(1024) char tsm_raw[];
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~uintptr_t(1023));
  char* sA = base;
  char* sB = base + TST * TA_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + TST * TB_BYTES);
  uint64_t* empty = full + TST;
  uint64_t* accf = empty + TST;  // [2]
  uint64_t* acce = accf + 2;     // [2]
  uint64_t* drain = acce + 2;    // MMA completion on the way out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (g.M + TBM - 1) / TBM, num_n = (g.N + TBN - 1) / TBN;
  const int tiles = num_m * num_n;
  const int num_k = (g.K + TBK - 1) / TBK;
  const int first_m = g.mode == MODE_AG ? (g.rank * g.rows_per_rank) / TBM : 0;
  const int parity = g.epoch & 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TST; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&accf[b], 1);
      tc::mbar_init(&acce[b], 4);
    }
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
    if (g.mode == MODE_AG && blockIdx.x == 0) {
      // announce "my shard for this epoch is in place" to every GPU
      for (int p = 0; p < g.world; ++p) st_release_sys(reinterpret_cast<int*>(g.peer_ready[p]) + g.rank, g.epoch);
    }
  }
  if (warp == 2) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto tile_mn = [&](int t, int& mt, int& nt) {
    nt = t % num_n;
    mt = (t / num_n + first_m) % num_m;
  };

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        int mt, nt;
        tile_mn(t, mt, nt);
        if (g.mode == MODE_AG && (mt * TBM) / g.rows_per_rank != g.rank) {
          if (!wait_geq<false>(g.block_flag + mt, g.epoch, g.err, 5)) { ok = false; break; }
          fence_proxy_async_global();
        }
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % TST;
          if (it >= TST && !tc::mbar_wait(&empty[s], ((it / TST) + 1) & 1, g.err, 1)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&full[s], TA_BYTES + TB_BYTES);
          tc::tma_load_2d(sA + s * TA_BYTES, &tmA, kt * TBK, mt * TBM, &full[s]);
          tc::tma_load_2d(sB + s * TB_BYTES, &tmB, kt * TBK, nt * TBN, &full[s]);
        }
      }
      if (!ok) {  // let the loads this thread issued land before the CTA can exit
        for (int j = max(0, it - TST); j < it; ++j) tc::mbar_wait_quiet(&full[j % TST], (j / TST) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      constexpr uint32_t idesc = tc::idesc_bf16_f32(TBM, TBN);
      int it = 0, i = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (i >= 2 && !tc::mbar_wait(&acce[buf], ((i >> 1) + 1) & 1, g.err, 6)) break;
        tc::tc_fence_after();
        bool ok = true;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % TST;
          if (!tc::mbar_wait(&full[s], (it / TST) & 1, g.err, 2)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t a_addr = tc::smem_u32(sA + s * TA_BYTES), b_addr = tc::smem_u32(sB + s * TB_BYTES);
#pragma unroll
          for (int kk = 0; kk < TBK / 16; ++kk)
            tc::mma_f16_ss(tmem + buf * TBN, tc::smem_desc_k_sw128(a_addr + kk * 32),
                           tc::smem_desc_k_sw128(b_addr + kk * 32), idesc, (kt | kk) != 0);
          tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(&accf[buf]);
        if (!ok) break;
      }
      tc::mma_commit(drain);
      tc::mbar_wait_quiet(drain, 0);  // every MMA of this CTA has completed
    }
  } else {
    // ---------------- epilogue warps 2..5 (128 threads)
    const int et = threadIdx.x - 64;  // 0..127
    const int lg = warp & 3;          // TMEM lane group this warp may access
    if (g.mode == MODE_AG) {
      // pull the remote row blocks assigned to this CTA
      const int blocks = g.M / TBM;
      for (int b = blockIdx.x; b < blocks; b += gridDim.x) {
        const int p = (b * TBM) / g.rows_per_rank;
        if (p == g.rank) continue;
        if (!wait_geq<true>(g.ready + p, g.epoch, g.err, 7)) break;
        const int r0 = b * TBM - p * g.rows_per_rank;
        const char* src = reinterpret_cast<const char*>(g.peer_a[p]) + (long long)r0 * g.K * 2;
        char* dst = reinterpret_cast<char*>(g.staging) + (long long)b * TBM * g.K * 2;
        const long long vecs = (long long)TBM * g.K / 8;
        for (long long v = et; v < vecs; v += 128) {
          const uint4 x = ld_v4(src + v * 16);  // plain load from the peer over NVLink
          *reinterpret_cast<uint4*>(dst + v * 16) = x;
        }
        fence_proxy_async_global();  // make the generic-proxy writes visible to TMA reads
        __threadfence();
        epi_bar();
        if (et == 0) st_release_gpu(g.block_flag + b, g.epoch);
      }
    }
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      int mt, nt;
      tile_mn(t, mt, nt);
      const int buf = i & 1;
      bool ok = tc::mbar_wait(&accf[buf], (i >> 1) & 1, g.err, 3);
      ok = __all_sync(0xffffffffu, ok) && __shfl_sync(0xffffffffu, *g.err, 0) == 0;
      tc::tc_fence_after();
      if (!ok) break;
      const int row = mt * TBM + lg * 32 + lane;
      __nv_bfloat16* dst_row = nullptr;
      if (row < g.M) {
        if (g.mode == MODE_RS) {
          const int owner = row / g.rows_per_rank, lr = row % g.rows_per_rank;
          __nv_bfloat16* recv = reinterpret_cast<__nv_bfloat16*>(g.peer_recv[owner]);
          dst_row = recv + (((long long)parity * g.world + g.rank) * g.rows_per_rank + lr) * g.N;
        } else {
          dst_row = g.c + (long long)row * g.ldc;
        }
      }
#pragma unroll 1
      for (int c = 0; c < TBN / 16; ++c) {
        uint32_t r[16];
        tc::tmem_ld16(tmem + buf * TBN + (static_cast<uint32_t>(lg * 32) << 16) + c * 16, r);
        tc::tmem_ld_wait();
        const int col = nt * TBN + c * 16;
        if (dst_row != nullptr && col < g.N) {
          __nv_bfloat16* cp = dst_row + col;
          if (col + 16 <= g.N) {
            uint4 o0 = make_uint4(pack_bf16x2(__uint_as_float(r[0]), __uint_as_float(r[1])),
                                  pack_bf16x2(__uint_as_float(r[2]), __uint_as_float(r[3])),
                                  pack_bf16x2(__uint_as_float(r[4]), __uint_as_float(r[5])),
                                  pack_bf16x2(__uint_as_float(r[6]), __uint_as_float(r[7])));
            uint4 o1 = make_uint4(pack_bf16x2(__uint_as_float(r[8]), __uint_as_float(r[9])),
                                  pack_bf16x2(__uint_as_float(r[10]), __uint_as_float(r[11])),
                                  pack_bf16x2(__uint_as_float(r[12]), __uint_as_float(r[13])),
                                  pack_bf16x2(__uint_as_float(r[14]), __uint_as_float(r[15])));
            reinterpret_cast<uint4*>(cp)[0] = o0;  // local, or a peer's receive slot (NVLink)
            reinterpret_cast<uint4*>(cp)[1] = o1;
          } else {
            for (int j = 0; j < 16 && col + j < g.N; ++j) cp[j] = __float2bfloat16(__uint_as_float(r[j]));
          }
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acce[buf]);
      if (g.mode == MODE_RS) {
        __threadfence_system();
        epi_bar();
        if (et == 0) {
          const int owner = (mt * TBM) / g.rows_per_rank, lb = (mt * TBM - owner * g.rows_per_rank) / TBM;
          red_add_release_sys(reinterpret_cast<int*>(g.peer_cnt[owner]) + 2 * lb + parity, 1);
        }
      }
    }
    if (g.mode == MODE_RS) {
      // reduce this GPU's row blocks once all partial tiles have arrived
      const int lblocks = g.rows_per_rank / TBM;
      const int target = g.world * num_n;
      for (int lb = blockIdx.x; lb < lblocks; lb += gridDim.x) {
        if (!wait_geq<true>(g.cnt + 2 * lb + parity, target, g.err, 8)) break;
        const long long vecs = (long long)TBM * g.N / 8;
        for (long long v = et; v < vecs; v += 128) {
          const long long e = (long long)lb * TBM * g.N + v * 8;
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int p = 0; p < g.world; ++p) {
            const uint4 x = *reinterpret_cast<const uint4*>(
                g.recv + ((long long)parity * g.world + p) * g.rows_per_rank * g.N + e);
            acc[0] += bf16_lo(x.x); acc[1] += bf16_hi(x.x); acc[2] += bf16_lo(x.y); acc[3] += bf16_hi(x.y);
            acc[4] += bf16_lo(x.z); acc[5] += bf16_hi(x.z); acc[6] += bf16_lo(x.w); acc[7] += bf16_hi(x.w);
          }
          *reinterpret_cast<uint4*>(g.out_rs + e) =
              make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                         pack_bf16x2(acc[6], acc[7]));
        }
        epi_bar();  // every thread is done with this block's receive slots
        if (et == 0) red_add_release_sys(g.cnt + 2 * lb + parity, -target);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 2) tc::tmem_dealloc(tmem, 512);
}

// ------------------------------------------------------------------------------- host
namespace {
void tp_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (ld * 2) % 16 == 0, "TMA alignment");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {TBK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult rc = cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                                             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(rc == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(rc));
}

int tp_grid(int tiles, int dev) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_tp_kernel, 192, TSMEM);
  return std::max(1, std::min(tiles, sms * std::max(1, per_sm)));
}
}  // namespace

// mode 0/1: out [M, N]; mode 2: out [rows_per_rank, N]. For AG/RS every pointer array is
// an int64 CUDA tensor of `world` addresses (this GPU's own buffers at index `rank`).
void gemm_tp(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t mode, int64_t rank, int64_t world,
             int64_t rows_per_rank, int64_t epoch, c10::optional<torch::Tensor> peer_a,
             c10::optional<torch::Tensor> staging, c10::optional<torch::Tensor> block_flag,
             c10::optional<torch::Tensor> ready, c10::optional<torch::Tensor> peer_ready,
             c10::optional<torch::Tensor> peer_recv, c10::optional<torch::Tensor> peer_cnt,
             c10::optional<torch::Tensor> recv, c10::optional<torch::Tensor> cnt, torch::Tensor err) {
  TORCH_CHECK(b.is_cuda() && b.scalar_type() == torch::kBFloat16 && b.stride(1) == 1, "b: bf16 [N, K] row-major");
  const int N = b.size(0), K = b.size(1);
  TpArgs g{};
  g.N = N;
  g.K = K;
  g.rank = static_cast<int>(rank);
  g.world = static_cast<int>(world);
  g.rows_per_rank = static_cast<int>(rows_per_rank);
  g.mode = static_cast<int>(mode);
  g.epoch = static_cast<int>(epoch);
  g.err = err.data_ptr<int>();
  const void* a_ptr;
  int64_t lda;
  if (mode == MODE_AG) {
    TORCH_CHECK(staging.has_value() && peer_a.has_value() && block_flag.has_value() && ready.has_value() &&
                    peer_ready.has_value(),
                "AG mode needs staging, peer_a, block_flag, ready, peer_ready");
    TORCH_CHECK(rows_per_rank % TBM == 0, "rows per rank must be a multiple of 128");
    g.M = static_cast<int>(world * rows_per_rank);
    // the local shard lives in staging already (rows rank*rows_per_rank ...)
    g.staging = reinterpret_cast<__nv_bfloat16*>(staging->data_ptr());
    g.peer_a = peer_a->data_ptr<int64_t>();
    g.block_flag = block_flag->data_ptr<int>();
    g.ready = ready->data_ptr<int>();
    g.peer_ready = peer_ready->data_ptr<int64_t>();
    a_ptr = staging->data_ptr();
    lda = K;
  } else {
    TORCH_CHECK(a.is_cuda() && a.scalar_type() == torch::kBFloat16 && a.stride(1) == 1 && a.size(1) == K,
                "a: bf16 [M, K] row-major");
    g.M = a.size(0);
    a_ptr = a.data_ptr();
    lda = a.stride(0);
  }
  if (mode == MODE_RS) {
    TORCH_CHECK(peer_recv.has_value() && peer_cnt.has_value() && recv.has_value() && cnt.has_value(),
                "RS mode needs peer_recv, peer_cnt, recv, cnt");
    TORCH_CHECK(g.M == world * rows_per_rank && rows_per_rank % TBM == 0 && N % 8 == 0, "RS shape");
    TORCH_CHECK(out.is_contiguous() && out.size(0) == rows_per_rank && out.size(1) == N, "RS out: [rows_per_rank, N]");
    TORCH_CHECK(recv->numel() >= 2 * world * rows_per_rank * N && cnt->numel() >= 2 * rows_per_rank / TBM,
                "RS receive buffers too small");
    g.peer_recv = peer_recv->data_ptr<int64_t>();
    g.peer_cnt = peer_cnt->data_ptr<int64_t>();
    g.recv = reinterpret_cast<__nv_bfloat16*>(recv->data_ptr());
    g.cnt = cnt->data_ptr<int>();
    g.out_rs = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  } else {
    TORCH_CHECK(out.size(0) == g.M && out.size(1) == N && out.stride(1) == 1, "out shape");
    g.c = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    g.ldc = out.stride(0);
  }
  if (g.M == 0 || N == 0) return;
  CUtensorMap ta, tb;
  tp_map(&ta, a_ptr, g.M, K, lda, TBM);
  tp_map(&tb, b.data_ptr(), N, K, b.stride(0), TBN);
  static bool attr = false;
  if (!attr) {
    AXR_CHECK_CUDA(cudaFuncSetAttribute(gemm_tp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TSMEM));
    attr = true;
  }
  const int tiles = ((g.M + TBM - 1) / TBM) * ((N + TBN - 1) / TBN);
  const int grid = tp_grid(tiles, b.device().index());
  void* args[] = {&ta, &tb, &g};
  AXR_CHECK_CUDA(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(gemm_tp_kernel), dim3(grid), dim3(192), args,
                                             TSMEM, at::cuda::getCurrentCUDAStream()));
}

}  // namespace axr
