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
#include "peer_sync.cuh"
#include "tc_common.cuh"

namespace axr {

__device__ __forceinline__ void comm_bar() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

constexpr int TBM = 128, TBN = 256, TBK = 64, TST = 4;
constexpr int TA_BYTES = TBM * TBK * 2, TB_BYTES = TBN * TBK * 2;
constexpr int EPI_COLS = 64;                      // epilogue staging width (columns per pass)
constexpr int STG_BYTES = 4 * 32 * EPI_COLS * 2;  // one [32 x 64] bf16 tile per epilogue warp
constexpr int TSMEM = 1024 + TST * (TA_BYTES + TB_BYTES) + STG_BYTES + 256;
constexpr int TP_THREADS = 320;
constexpr int AG_CH = 8;   // a remote 128-row block is pulled as 8 chunks of 16 rows
constexpr int RS_CH = 16;  // an owned 128-row block is reduced as 16 chunks of 8 rows
constexpr int RS_MAXW = 8;  // partials loaded together per reduction step
constexpr int MODE_PLAIN = 0, MODE_AG = 1, MODE_RS = 2;

struct TpArgs {
  __nv_bfloat16* c;  // PLAIN/AG output [M, N]
  long long ldc;
  int M, N, K;
  int rank, world, rows_per_rank;  // AG/RS: M = world * rows_per_rank
  int mode;
  int epoch;  // 1, 2, 3, ... per call of this mode on this communicator (same on every GPU)
  unsigned long long wait_ns;  // bound of every wait in this kernel (peer-dependent)
  // AG
  const int64_t* peer_a;  // [world] base addresses of the peers' A shards [rows_per_rank, K]
  __nv_bfloat16* staging;   // local [M, K]; the TMA map of A covers it
  int* flags;               // AG: [M/128][AG_CH] epoch of each pulled chunk; RS: [rows/128][2] chunks reduced
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

// Thread 0 of the comm warps waits; the outcome reaches all 128 comm threads through
// shared memory and the barrier, so the four warps always take the same branch.
__device__ __forceinline__ bool comm_wait(const int* p, int target, volatile int* err, int code, int ct,
                                          volatile int* shared_ok, unsigned long long limit) {
  if (ct == 0) *shared_ok = wait_geq<true>(p, target, err, code, limit) ? 1 : 0;
  comm_bar();
  const bool ok = *shared_ok != 0;
  comm_bar();  // nobody overwrites shared_ok before everyone has read it
  return ok;
}

// Tile t -> (m-block, n-block). Tiles run in groups of GROUP_M row blocks with the row
// block varying fastest inside a group, so the CTAs in flight share both their A rows and
// their B columns through L2 (B is streamed from HBM about M / (128 * GROUP_M) times).
// The row-block ordinal o maps to a row block per mode. AG: this GPU's own row blocks
// first, then the remote ones in the order they are pulled. RS: every GPU walks the row
// blocks in the same interleaved order (block j of owner 0, of owner 1, ...), so block j
// of every owner completes at about the same time and its reduction overlaps the GEMM of
// the blocks after it.
constexpr int GROUP_M = 16;
__device__ __forceinline__ void tp_tile(const TpArgs& g, int t, int num_n, int num_m, int first_m, int& mt,
                                        int& nt) {
  const int group = GROUP_M * num_n;
  const int first_o = (t / group) * GROUP_M;
  const int gm = min(num_m - first_o, GROUP_M);
  const int in = t - (t / group) * group;
  const int o = first_o + in % gm;
  nt = in / gm;
  if (g.mode == MODE_AG) {
    mt = (o + first_m) % num_m;
  } else if (g.mode == MODE_RS) {
    const int lblocks = g.rows_per_rank / TBM;
    mt = (o % g.world) * lblocks + o / g.world;
  } else {
    mt = o;
  }
}

// Roles (320 threads): warp 0 TMA producer, warp 1 MMA issuer (and TMEM owner: warp 2),
// warps 2-5 epilogue (TMEM lane group = warp % 4), warps 6-9 communication (AG pulls of
// peer rows, RS reduction of the partial tiles received).
__global__ void __launch_bounds__(TP_THREADS, 1) gemm_tp_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                const __grid_constant__ CUtensorMap tmB, TpArgs g) {
  extern __shared__ __align__(1024) char tsm_raw[];
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(tsm_raw) + 1023) & ~uintptr_t(1023));
  char* sA = base;
  char* sB = base + TST * TA_BYTES;
  char* stg = sB + TST * TB_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(stg + STG_BYTES);
  uint64_t* empty = full + TST;
  uint64_t* accf = empty + TST;  // [2]
  uint64_t* acce = accf + 2;     // [2]
  uint64_t* drain = acce + 2;    // MMA completion on the way out
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* comm_ok = reinterpret_cast<volatile int*>(tmem_slot + 1);

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

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        int mt, nt;
        tp_tile(g, t, num_n, num_m, first_m, mt, nt);
        if (g.mode == MODE_AG && (mt * TBM) / g.rows_per_rank != g.rank) {
          for (int ch = 0; ok && ch < AG_CH; ++ch) ok = wait_geq<false>(g.flags + mt * AG_CH + ch, g.epoch, g.err, 5, g.wait_ns);
          if (!ok) break;
          fence_proxy_async_global();  // order the TMA reads after the pulled rows
        }
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % TST;
          if (it >= TST && !tc::mbar_wait(&empty[s], ((it / TST) + 1) & 1, g.err, 1, g.wait_ns)) { ok = false; break; }
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
        if (i >= 2 && !tc::mbar_wait(&acce[buf], ((i >> 1) + 1) & 1, g.err, 6, g.wait_ns)) break;
        tc::tc_fence_after();
        bool ok = true;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % TST;
          if (!tc::mbar_wait(&full[s], (it / TST) & 1, g.err, 2, g.wait_ns)) { ok = false; break; }
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
  } else if (warp < 6) {
    // ---------------- epilogue warps 2..5: TMEM -> registers -> bf16 -> shared staging -> coalesced stores
    const int lg = warp & 3;  // TMEM lane group this warp may access
    char* my_stg = stg + (warp - 2) * (32 * EPI_COLS * 2);
    const bool vec_ok = g.mode == MODE_RS || (g.ldc & 7) == 0;
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      int mt, nt;
      tp_tile(g, t, num_n, num_m, first_m, mt, nt);
      const int buf = i & 1;
      bool ok = tc::mbar_wait(&accf[buf], (i >> 1) & 1, g.err, 3, g.wait_ns);
      ok = __all_sync(0xffffffffu, ok) && __shfl_sync(0xffffffffu, *g.err, 0) == 0;
      tc::tc_fence_after();
      if (!ok) break;
#pragma unroll 1
      for (int cg = 0; cg < TBN / EPI_COLS; ++cg) {
        uint32_t r[4][16];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          tc::tmem_ld16(tmem + buf * TBN + (static_cast<uint32_t>(lg * 32) << 16) + cg * EPI_COLS + c * 16, r[c]);
        tc::tmem_ld_wait();
        if (cg == TBN / EPI_COLS - 1) {  // accumulator buffer fully read: hand it back to the MMA warp
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&acce[buf]);
        }
        // this lane's row -> staging, 16-byte granules XOR-swizzled by row to avoid bank conflicts
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t* v = &r[c][h * 8];
            const uint4 o = make_uint4(pack_bf16x2(__uint_as_float(v[0]), __uint_as_float(v[1])),
                                       pack_bf16x2(__uint_as_float(v[2]), __uint_as_float(v[3])),
                                       pack_bf16x2(__uint_as_float(v[4]), __uint_as_float(v[5])),
                                       pack_bf16x2(__uint_as_float(v[6]), __uint_as_float(v[7])));
            const int gidx = (c * 2 + h) ^ (lane & 7);
            *reinterpret_cast<uint4*>(my_stg + lane * 128 + gidx * 16) = o;
          }
        }
        __syncwarp();
        // 32 rows x 128 bytes: 8 lanes write one row's 128 contiguous bytes
#pragma unroll
        for (int it2 = 0; it2 < 8; ++it2) {
          const int rr = it2 * 4 + (lane >> 3), gq = lane & 7;
          const uint4 v = *reinterpret_cast<const uint4*>(my_stg + rr * 128 + ((gq ^ (rr & 7)) * 16));
          const int row = mt * TBM + lg * 32 + rr;
          const int col = nt * TBN + cg * EPI_COLS + gq * 8;
          if (row < g.M && col < g.N) {
            __nv_bfloat16* dst;
            if (g.mode == MODE_RS) {
              const int owner = row / g.rows_per_rank, lr = row - owner * g.rows_per_rank;
              dst = reinterpret_cast<__nv_bfloat16*>(g.peer_recv[owner]) +
                    (((long long)parity * g.world + g.rank) * g.rows_per_rank + lr) * g.N + col;
            } else {
              dst = g.c + (long long)row * g.ldc + col;
            }
            if (vec_ok && col + 8 <= g.N) {
              *reinterpret_cast<uint4*>(dst) = v;  // local, or a peer's receive slot (NVLink)
            } else {
              const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
              for (int j = 0; j < 8 && col + j < g.N; ++j) dst[j] = e[j];
            }
          }
        }
        __syncwarp();
      }
      if (g.mode == MODE_RS) {
        // this warp's 32 rows of the partial tile are out: count them at the owner
        __threadfence_system();
        __syncwarp();
        if (lane == 0) {
          const int owner = (mt * TBM) / g.rows_per_rank, lb = (mt * TBM - owner * g.rows_per_rank) / TBM;
          red_add_release_sys(reinterpret_cast<int*>(g.peer_cnt[owner]) + 2 * lb + parity, 1);
        }
      }
    }
  } else {
    // ---------------- communication warps 6..9 (128 threads)
    const int ct = threadIdx.x - 192;
    if (g.mode == MODE_AG) {
      // pull remote 16-row chunks, in the order the tiles consume them
      const int nb = g.M / TBM, lbk = g.rows_per_rank / TBM;
      const int items = (nb - lbk) * AG_CH;
      const long long vecs = 16LL * g.K / 8;  // 16-byte vectors per chunk (16 rows x K)
      for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int b = (first_m + lbk + item / AG_CH) % nb, ch = item % AG_CH;
        const int p = (b * TBM) / g.rows_per_rank;
        if (!comm_wait(g.ready + p, g.epoch, g.err, 7, ct, comm_ok, g.wait_ns)) break;
        const long long r0 = (long long)b * TBM - (long long)p * g.rows_per_rank + ch * 16;
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(g.peer_a[p]) + r0 * g.K * 2);
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(g.staging) +
                                              ((long long)b * TBM + ch * 16) * g.K * 2);
        for (long long v = ct; v < vecs; v += 128 * 8) {
          uint4 x[8];
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (v + u * 128 < vecs) x[u] = src[v + u * 128];  // peer memory over NVLink, 8 loads in flight
#pragma unroll
          for (int u = 0; u < 8; ++u)
            if (v + u * 128 < vecs) dst[v + u * 128] = x[u];
        }
        fence_proxy_async_global();  // the TMA (async proxy) reads these rows next
        __threadfence();
        comm_bar();
        if (ct == 0) st_release_gpu(g.flags + b * AG_CH + ch, g.epoch);
      }
    } else if (g.mode == MODE_RS) {
      // reduce this GPU's rows, 8-row chunks, as soon as all partial tiles of a block are in
      const int lbk = g.rows_per_rank / TBM;
      const int items = lbk * RS_CH;
      const int target = g.world * num_n * 4;  // one arrival per epilogue warp per tile
      const long long vecs = 8LL * g.N / 8;     // 16-byte vectors per chunk (8 rows x N)
      const long long slot = (long long)g.rows_per_rank * g.N;
      const __nv_bfloat16* rbase = g.recv + (long long)parity * g.world * slot;
      for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int lb = item / RS_CH, ch = item % RS_CH;
        if (!comm_wait(g.cnt + 2 * lb + parity, target, g.err, 8, ct, comm_ok, g.wait_ns)) break;
        const long long e0 = ((long long)lb * TBM + ch * 8) * g.N;
        // every partial of a vector is loaded before any is summed (up to 8 GPUs x 2 vectors
        // in flight per thread): the reduction is bound by memory-level parallelism
        for (long long v = ct; v < vecs; v += 128 * 2) {
          float acc[2][8];
#pragma unroll
          for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[u][j] = 0.f;
          for (int p0 = 0; p0 < g.world; p0 += RS_MAXW) {
            uint4 x[RS_MAXW][2];
#pragma unroll
            for (int q = 0; q < RS_MAXW; ++q)
#pragma unroll
              for (int u = 0; u < 2; ++u)
                if (p0 + q < g.world && v + u * 128 < vecs)
                  x[q][u] = *reinterpret_cast<const uint4*>(rbase + (p0 + q) * slot + e0 + (v + u * 128) * 8);
#pragma unroll
            for (int q = 0; q < RS_MAXW; ++q) {
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                if (p0 + q < g.world && v + u * 128 < vecs) {
                  acc[u][0] += bf16_lo(x[q][u].x); acc[u][1] += bf16_hi(x[q][u].x);
                  acc[u][2] += bf16_lo(x[q][u].y); acc[u][3] += bf16_hi(x[q][u].y);
                  acc[u][4] += bf16_lo(x[q][u].z); acc[u][5] += bf16_hi(x[q][u].z);
                  acc[u][6] += bf16_lo(x[q][u].w); acc[u][7] += bf16_hi(x[q][u].w);
                }
              }
            }
          }
#pragma unroll
          for (int u = 0; u < 2; ++u)
            if (v + u * 128 < vecs)
              *reinterpret_cast<uint4*>(g.out_rs + e0 + (v + u * 128) * 8) =
                  make_uint4(pack_bf16x2(acc[u][0], acc[u][1]), pack_bf16x2(acc[u][2], acc[u][3]),
                             pack_bf16x2(acc[u][4], acc[u][5]), pack_bf16x2(acc[u][6], acc[u][7]));
        }
        comm_bar();  // every comm thread is done with this chunk's receive slots
        if (ct == 0) {
          // the last chunk of a block takes the block's arrivals back off its counter
          if (atomicAdd(g.flags + 2 * lb + parity, 1) == RS_CH - 1) {
            g.flags[2 * lb + parity] = 0;
            red_add_release_sys(g.cnt + 2 * lb + parity, -target);
          }
        }
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

int tp_grid(int work, int dev) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_tp_kernel, TP_THREADS, TSMEM);
  return std::max(1, std::min(work, sms * std::max(1, per_sm)));
}
}  // namespace

// mode 0/1: out [M, N]; mode 2: out [rows_per_rank, N]. For AG/RS every pointer array is
// an int64 CUDA tensor of `world` addresses (this GPU's own buffers at index `rank`).
// flags: AG int32 [M/128 * 8] chunk epochs (zero-initialised once); RS int32
// [rows_per_rank/128 * 2] reduce-done counters (zero-initialised once).
void gemm_tp(torch::Tensor a, torch::Tensor b, torch::Tensor out, int64_t mode, int64_t rank, int64_t world,
             int64_t rows_per_rank, int64_t epoch, c10::optional<torch::Tensor> peer_a,
             c10::optional<torch::Tensor> staging, c10::optional<torch::Tensor> flags,
             c10::optional<torch::Tensor> ready, c10::optional<torch::Tensor> peer_ready,
             c10::optional<torch::Tensor> peer_recv, c10::optional<torch::Tensor> peer_cnt,
             c10::optional<torch::Tensor> recv, c10::optional<torch::Tensor> cnt, torch::Tensor err) {
  TORCH_CHECK(b.is_cuda() && b.scalar_type() == torch::kBFloat16 && b.stride(1) == 1, "b: bf16 [N, K] row-major");
  TORCH_CHECK(err.is_cuda() && err.scalar_type() == torch::kInt32, "err: int32 CUDA tensor");
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
  g.wait_ns = peer_wait_ns();
  const void* a_ptr;
  int64_t lda;
  int comm_items = 0;
  if (mode == MODE_AG) {
    TORCH_CHECK(staging.has_value() && peer_a.has_value() && flags.has_value() && ready.has_value() &&
                    peer_ready.has_value(),
                "AG mode needs staging, peer_a, flags, ready, peer_ready");
    TORCH_CHECK(rows_per_rank % TBM == 0 && K % 8 == 0, "AG: rows per rank must be a multiple of 128, K of 8");
    g.M = static_cast<int>(world * rows_per_rank);
    TORCH_CHECK(staging->numel() >= static_cast<int64_t>(g.M) * K && flags->numel() >= (g.M / TBM) * AG_CH,
                "AG buffers too small");
    // the local shard lives in staging already (rows rank*rows_per_rank ...)
    g.staging = reinterpret_cast<__nv_bfloat16*>(staging->data_ptr());
    g.peer_a = peer_a->data_ptr<int64_t>();
    g.flags = flags->data_ptr<int>();
    g.ready = ready->data_ptr<int>();
    g.peer_ready = peer_ready->data_ptr<int64_t>();
    a_ptr = staging->data_ptr();
    lda = K;
    comm_items = (g.M / TBM - static_cast<int>(rows_per_rank) / TBM) * AG_CH;
  } else {
    TORCH_CHECK(a.is_cuda() && a.scalar_type() == torch::kBFloat16 && a.stride(1) == 1 && a.size(1) == K,
                "a: bf16 [M, K] row-major");
    g.M = a.size(0);
    a_ptr = a.data_ptr();
    lda = a.stride(0);
  }
  if (mode == MODE_RS) {
    TORCH_CHECK(peer_recv.has_value() && peer_cnt.has_value() && recv.has_value() && cnt.has_value() &&
                    flags.has_value(),
                "RS mode needs peer_recv, peer_cnt, recv, cnt, flags");
    TORCH_CHECK(g.M == world * rows_per_rank && rows_per_rank % TBM == 0 && N % 8 == 0, "RS shape");
    TORCH_CHECK(out.is_contiguous() && out.size(0) == rows_per_rank && out.size(1) == N, "RS out: [rows_per_rank, N]");
    TORCH_CHECK(recv->numel() >= 2 * world * rows_per_rank * N && cnt->numel() >= 2 * rows_per_rank / TBM &&
                    flags->numel() >= 2 * rows_per_rank / TBM,
                "RS buffers too small");
    g.peer_recv = peer_recv->data_ptr<int64_t>();
    g.peer_cnt = peer_cnt->data_ptr<int64_t>();
    g.recv = reinterpret_cast<__nv_bfloat16*>(recv->data_ptr());
    g.cnt = cnt->data_ptr<int>();
    g.flags = flags->data_ptr<int>();
    g.out_rs = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    comm_items = static_cast<int>(rows_per_rank / TBM) * RS_CH;
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
  const int grid = tp_grid(std::max(tiles, comm_items), b.device().index());
  void* args[] = {&ta, &tb, &g};
  AXR_CHECK_CUDA(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(gemm_tp_kernel), dim3(grid), dim3(TP_THREADS),
                                             args, TSMEM, at::cuda::getCurrentCUDAStream()));
}

}  // namespace axr
