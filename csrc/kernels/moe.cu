// Expert-parallel mixture-of-experts: all-to-all dispatch -> grouped expert GEMMs on
// the tcgen05 tensor cores -> all-to-all combine, with the transfers issued from inside
// the kernels as peer (NVLink) stores.
//
// Each GPU owns E_l experts. One MoE layer call (epoch e, the same on every GPU):
//
//  1. moe_dispatch_kernel (cooperative): every (token, k) pair gets a position within
//     its (destination GPU, local expert) group; each GPU publishes its count matrix to
//     every peer (system-scope release), waits for all peers' counts, derives where its
//     rows go in each destination's expert-sorted receive buffer (every expert region
//     padded to 128 rows) and stores the token rows there over NVLink, with the origin
//     (GPU, slot) and routing weight of each row. The last CTA to finish raises this
//     GPU's arrival flag on every destination.
//  2. moe_gemm_kernel, gate/up: persistent grouped GEMM over the received rows, B = the
//     expert's fused gate/up weights (rows interleaved in blocks of 128 gate / 128 up),
//     SwiGLU applied in the epilogue (TMEM -> registers), output h. The TMA producer of a
//     row block first waits (bounded) for the arrival flags of the source GPUs whose
//     rows fall in that block, so blocks of early sources (and of this GPU) start while
//     later sources' rows are still crossing NVLink.
//  3. moe_gemm_kernel, down: grouped GEMM h x W2^T; the epilogue scales each row by its
//     routing weight and stores it straight into the origin GPU's combine slot
//     [token, k] (coalesced 128-byte row segments over NVLink). The last CTA raises this
//     GPU's "combined" flag on every origin.
//  4. moe_combine_kernel (origin): waits for every expert GPU's flag, sums the k slots.
//
// No TMA reads peer memory and no multicast is used; every wait is bounded and reports
// through the error flag. The reference has no MoE support at all (no expert code).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include "common.cuh"
#include "peer_sync.cuh"
#include "tc_common.cuh"

namespace axr {
namespace moe {

constexpr int BM = 128, BN = 256, BK = 64, ST = 4;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
constexpr int EPI_COLS = 64;
constexpr int STG_BYTES = 4 * 32 * EPI_COLS * 2;
constexpr int SMEM = 1024 + ST * (A_BYTES + B_BYTES) + STG_BYTES + 1024;
constexpr int THREADS = 192;
constexpr int MAXW = 8, MAXE = 64;
constexpr int GROUP_M = 16;

// ------------------------------------------------------------------------------ dispatch
struct DispatchArgs {
  const __nv_bfloat16* x;  // [T, H]
  const int* topk_idx;     // [T, K] global expert ids
  const float* topk_w;     // [T, K]
  int T, K, H, E_l, rank, world, epoch, cap_rows;
  int* pair_pos;           // [T*K]
  int* gcount;             // [world*E_l], zero on entry; zeroed again by the last CTA
  int* grid_bar;           // [2], zero on entry; reset by the last CTA
  const int64_t* peer_cnt_all;   // [world] -> int [world src][world dst][E_l]
  const int64_t* peer_cnt_flag;  // [world] -> int [world src]
  const int* cnt_all;
  const int* cnt_flag;
  const int64_t* peer_recv_x;     // [world] -> bf16 [cap_rows, H]
  const int64_t* peer_recv_meta;  // [world] -> int2 [cap_rows] (origin gpu, origin slot)
  const int64_t* peer_recv_w;     // [world] -> float [cap_rows]
  const int64_t* peer_arr_flag;   // [world] -> int [world src]
  volatile int* err;
  unsigned long long wait_ns;
};

__device__ __forceinline__ bool cta_wait_all(const int* flags, int n, int target, volatile int* err, int code,
                                             int* s_ok, unsigned long long limit) {
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int s = 0; ok && s < n; ++s) ok = wait_geq<true>(flags + s, target, err, code, limit);
    *s_ok = ok ? 1 : 0;
  }
  __syncthreads();
  const bool ok = *s_ok != 0;
  __syncthreads();
  return ok;
}

__global__ void __launch_bounds__(256) moe_dispatch_kernel(DispatchArgs a) {
  __shared__ int s_ok;
  __shared__ int s_base[MAXW * MAXE];
  const int W = a.world, El = a.E_l, pairs = a.T * a.K;
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x, gthreads = gridDim.x * blockDim.x;
  // 1. position of every pair within its (destination, expert) group
  for (int i = gtid; i < pairs; i += gthreads) {
    const int eg = a.topk_idx[i];
    if (eg < 0 || eg >= W * El) {  // invalid expert id: record and drop the pair
      atomicCAS(const_cast<int*>(a.err), 0, 30);
      a.pair_pos[i] = -1;
      continue;
    }
    a.pair_pos[i] = atomicAdd(&a.gcount[eg], 1);  // eg = dst * E_l + e
  }
  // grid barrier (cooperative launch: every CTA is resident)
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    atomicAdd(&a.grid_bar[0], 1);
    s_ok = wait_geq<false>(&a.grid_bar[0], gridDim.x, a.err, 31, a.wait_ns) ? 1 : 0;
  }
  __syncthreads();
  if (!s_ok) return;
  // 2. CTA 0 publishes this GPU's counts [dst][e] to every peer
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < W * W * El; i += blockDim.x) {
      const int p = i / (W * El), r = i % (W * El);
      int* dst = reinterpret_cast<int*>(a.peer_cnt_all[p]) + a.rank * W * El + r;
      *dst = ld_acquire_gpu(&a.gcount[r]);
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0)
      for (int p = 0; p < W; ++p) st_release_sys(reinterpret_cast<int*>(a.peer_cnt_flag[p]) + a.rank, a.epoch);
  }
  // 3. every CTA: wait for all sources' counts, derive this GPU's base row per (dst, e)
  if (!cta_wait_all(a.cnt_flag, W, a.epoch, a.err, 32, &s_ok, a.wait_ns)) return;
  if (threadIdx.x < W) {
    const int d = threadIdx.x;
    int off = 0;
    for (int e = 0; e < El; ++e) {
      int tot = 0, before = 0;
      for (int s = 0; s < W; ++s) {
        const int c = a.cnt_all[(s * W + d) * El + e];
        tot += c;
        if (s < a.rank) before += c;
      }
      s_base[d * El + e] = off + before;
      off += (tot + BM - 1) / BM * BM;
    }
  }
  __syncthreads();
  // 4. push rows: one warp per pair, 16-byte stores into the destination's buffer
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gwarp = blockIdx.x * (blockDim.x >> 5) + warp, nwarps = gridDim.x * (blockDim.x >> 5);
  const int vecs = a.H / 8;
  for (int i = gwarp; i < pairs; i += nwarps) {
    const int eg = a.topk_idx[i];
    if (a.pair_pos[i] < 0 || eg < 0 || eg >= W * El) continue;
    const int d = eg / El, e = eg % El;
    const int row = s_base[d * El + e] + a.pair_pos[i];
    if (row >= a.cap_rows) {
      if (lane == 0) atomicCAS(const_cast<int*>(a.err), 0, 33);
      continue;
    }
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (long long)(i / a.K) * a.H);
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.peer_recv_x[d]) + (long long)row * a.H);
    for (int v = lane; v < vecs; v += 32 * 4) {
      uint4 t[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v + u * 32 < vecs) t[u] = src[v + u * 32];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (v + u * 32 < vecs) dst[v + u * 32] = t[u];
    }
    if (lane == 0) {
      reinterpret_cast<int2*>(a.peer_recv_meta[d])[row] = make_int2(a.rank, i);
      reinterpret_cast<float*>(a.peer_recv_w[d])[row] = a.topk_w[i];
    }
  }
  // 5. the last CTA to finish raises this GPU's arrival flag on every destination
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(&a.grid_bar[1], 1) == gridDim.x - 1) {
      __threadfence_system();
      for (int p = 0; p < W; ++p) st_release_sys(reinterpret_cast<int*>(a.peer_arr_flag[p]) + a.rank, a.epoch);
      for (int r = 0; r < W * El; ++r) a.gcount[r] = 0;
      a.grid_bar[0] = 0;
      a.grid_bar[1] = 0;
    }
  }
}

// ------------------------------------------------------------------------------ grouped GEMM
struct GemmArgs {
  int mode;  // 0: gate/up + SwiGLU -> h ; 1: down -> combine into the origins
  int rank, world, E_l, N, K, epoch, cap_rows;
  const int* cnt_all;   // local [world src][world dst][E_l]
  const int* cnt_flag;  // local [world]
  const int* arr_flag;  // local [world]
  __nv_bfloat16* h;     // mode 0 output [cap_rows, N/2]
  long long ldh;
  // mode 1
  const int2* recv_meta;
  const float* recv_w;
  const int64_t* peer_comb;       // [world] -> bf16 [slots, N]
  const int64_t* peer_comb_flag;  // [world] -> int [world]
  int* done_ctr;                  // local counter, zero on entry; reset by the last CTA
  volatile int* err;
  unsigned long long wait_ns;
};

struct TileMap {
  int tot[MAXE], roff[MAXE], mb0[MAXE + 1];
  int soff[MAXE][MAXW + 1];  // start of source s's rows inside the expert region
  int total_mb;
};

__device__ __forceinline__ int expert_of(const TileMap& tm, int El, int mb) {
  int e = 0;
  while (e + 1 < El && tm.mb0[e + 1] <= mb) ++e;
  return e;
}

__global__ void __launch_bounds__(THREADS, 1) moe_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                              const __grid_constant__ CUtensorMap tmB, GemmArgs g) {
  extern __shared__ __align__(1024) char sm_raw[];
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) & ~uintptr_t(1023));
  char* sA = base;
  char* sB = sA + ST * A_BYTES;
  char* stg = sB + ST * B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(stg + STG_BYTES);
  uint64_t* empty = full + ST;
  uint64_t* accf = empty + ST;
  uint64_t* acce = accf + 2;
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* s_ok = reinterpret_cast<int*>(tmem_slot + 1);
  __shared__ TileMap tm;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = g.world, El = g.E_l;
  // ---- tile map from the count matrix (wait until every source has published it)
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int s = 0; ok && s < W; ++s) ok = wait_geq<true>(g.cnt_flag + s, g.epoch, g.err, 41, g.wait_ns);
    *s_ok = ok ? 1 : 0;
    if (ok) {
      int off = 0, mb = 0;
      for (int e = 0; e < El; ++e) {
        int t = 0;
        for (int s = 0; s < W; ++s) {
          tm.soff[e][s] = t;
          t += g.cnt_all[(s * W + g.rank) * El + e];
        }
        tm.soff[e][W] = t;
        tm.tot[e] = t;
        tm.roff[e] = off;
        tm.mb0[e] = mb;
        const int nb = (t + BM - 1) / BM;
        off += nb * BM;
        mb += nb;
      }
      tm.mb0[El] = mb;
      tm.total_mb = mb;
      if (off > g.cap_rows) {
        atomicCAS(const_cast<int*>(g.err), 0, 42);
        *s_ok = 0;
      }
    }
    tc::mbar_init(drain, 1);
    for (int s = 0; s < ST; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&accf[b], 1);
      tc::mbar_init(&acce[b], 4);
    }
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
  }
  if (warp == 2) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const bool map_ok = *s_ok != 0;
  const int num_n = g.N / BN, num_k = g.K / BK;
  const int tiles = map_ok ? tm.total_mb * num_n : 0;

  auto tile_of = [&](int t, int& mb, int& nt) {
    const int group = GROUP_M * num_n;
    const int first = (t / group) * GROUP_M;
    const int gm = min(tm.total_mb - first, GROUP_M);
    const int in = t - (t / group) * group;
    mb = first + in % gm;
    nt = in / gm;
  };

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int it = 0;
      bool ok = true;
      uint32_t arrived = 0;  // bitmask of sources whose rows are known to have landed
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        int mb, nt;
        tile_of(t, mb, nt);
        const int e = expert_of(tm, El, mb);
        const int r0 = (mb - tm.mb0[e]) * BM;  // row inside the expert region
        if (g.mode == 0) {
          for (int s = 0; ok && s < W; ++s) {
            if (arrived >> s & 1) continue;
            if (tm.soff[e][s + 1] <= r0 || tm.soff[e][s] >= r0 + BM) continue;  // no rows of s here
            ok = wait_geq<true>(g.arr_flag + s, g.epoch, g.err, 43, g.wait_ns);
            if (ok) arrived |= 1u << s;
          }
          if (!ok) break;
          fence_proxy_async_global();  // peer-written rows -> TMA (async proxy) reads
        }
        const int ya = tm.roff[e] + r0, yb = e * g.N + nt * BN;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % ST;
          if (it >= ST && !tc::mbar_wait(&empty[s], ((it / ST) + 1) & 1, g.err, 44, g.wait_ns)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES);
          tc::tma_load_2d(sA + s * A_BYTES, &tmA, kt * BK, ya, &full[s]);
          tc::tma_load_2d(sB + s * B_BYTES, &tmB, kt * BK, yb, &full[s]);
        }
      }
      if (!ok) {
        for (int j = max(0, it - ST); j < it; ++j) tc::mbar_wait_quiet(&full[j % ST], (j / ST) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN);
      int it = 0, i = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (i >= 2 && !tc::mbar_wait(&acce[buf], ((i >> 1) + 1) & 1, g.err, 45, g.wait_ns)) break;
        tc::tc_fence_after();
        bool ok = true;
        for (int kt = 0; kt < num_k; ++kt, ++it) {
          const int s = it % ST;
          if (!tc::mbar_wait(&full[s], (it / ST) & 1, g.err, 46, g.wait_ns)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t a_addr = tc::smem_u32(sA + s * A_BYTES), b_addr = tc::smem_u32(sB + s * B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            tc::mma_f16_ss(tmem + buf * BN, tc::smem_desc_k_sw128(a_addr + kk * 32),
                           tc::smem_desc_k_sw128(b_addr + kk * 32), idesc, (kt | kk) != 0);
          tc::mma_commit(&empty[s]);
        }
        tc::mma_commit(&accf[buf]);
        if (!ok) break;
      }
      tc::mma_commit(drain);
      tc::mbar_wait_quiet(drain, 0);
    }
  } else {
    // ---------------- epilogue warps 2..5
    const int lg = warp & 3;
    char* my_stg = stg + (warp - 2) * (32 * EPI_COLS * 2);
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      int mb, nt;
      tile_of(t, mb, nt);
      const int e = expert_of(tm, El, mb);
      const int r0 = (mb - tm.mb0[e]) * BM;
      const int buf = i & 1;
      bool ok = tc::mbar_wait(&accf[buf], (i >> 1) & 1, g.err, 47, g.wait_ns);
      ok = __all_sync(0xffffffffu, ok) && __shfl_sync(0xffffffffu, *g.err, 0) == 0;
      tc::tc_fence_after();
      if (!ok) break;
      const uint32_t tbase = tmem + buf * BN + (static_cast<uint32_t>(lg * 32) << 16);
      const int passes = g.mode == 0 ? 2 : 4;  // gate/up: 128 output columns; down: 256
#pragma unroll 1
      for (int cg = 0; cg < passes; ++cg) {
        uint32_t r[4][16];
        if (g.mode == 0) {
          uint32_t u[4][16];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            tc::tmem_ld16(tbase + cg * EPI_COLS + c * 16, r[c]);        // gate columns
            tc::tmem_ld16(tbase + 128 + cg * EPI_COLS + c * 16, u[c]);  // up columns
          }
          tc::tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float gt = __uint_as_float(r[c][j]);
              r[c][j] = __float_as_uint(gt / (1.f + __expf(-gt)) * __uint_as_float(u[c][j]));
            }
        } else {
#pragma unroll
          for (int c = 0; c < 4; ++c) tc::tmem_ld16(tbase + cg * EPI_COLS + c * 16, r[c]);
          tc::tmem_ld_wait();
          const int lr = r0 + lg * 32 + lane;
          const float w = lr < tm.tot[e] ? g.recv_w[tm.roff[e] + lr] : 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int j = 0; j < 16; ++j) r[c][j] = __float_as_uint(__uint_as_float(r[c][j]) * w);
        }
        if (cg == passes - 1) {
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(&acce[buf]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const uint32_t* v = &r[c][hh * 8];
            const uint4 o = make_uint4(pack_bf16x2(__uint_as_float(v[0]), __uint_as_float(v[1])),
                                       pack_bf16x2(__uint_as_float(v[2]), __uint_as_float(v[3])),
                                       pack_bf16x2(__uint_as_float(v[4]), __uint_as_float(v[5])),
                                       pack_bf16x2(__uint_as_float(v[6]), __uint_as_float(v[7])));
            *reinterpret_cast<uint4*>(my_stg + lane * 128 + (((c * 2 + hh) ^ (lane & 7)) * 16)) = o;
          }
        __syncwarp();
#pragma unroll
        for (int it2 = 0; it2 < 8; ++it2) {
          const int rr = it2 * 4 + (lane >> 3), gq = lane & 7;
          const uint4 v = *reinterpret_cast<const uint4*>(my_stg + rr * 128 + ((gq ^ (rr & 7)) * 16));
          const int lr = r0 + lg * 32 + rr;  // row inside the expert region
          if (lr < tm.tot[e]) {
            const int row = tm.roff[e] + lr;
            if (g.mode == 0) {
              const int col = nt * (BN / 2) + cg * EPI_COLS + gq * 8;
              *reinterpret_cast<uint4*>(g.h + (long long)row * g.ldh + col) = v;
            } else {
              const int col = nt * BN + cg * EPI_COLS + gq * 8;
              const int2 m = g.recv_meta[row];
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(g.peer_comb[m.x]) + (long long)m.y * g.N + col;
              *reinterpret_cast<uint4*>(dst) = v;  // origin GPU's combine slot (NVLink when remote)
            }
          }
        }
        __syncwarp();
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 2) tc::tmem_dealloc(tmem, 512);
  if (g.mode == 1 && threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(g.done_ctr, 1) == gridDim.x - 1) {  // last CTA: every combine row is out
      __threadfence_system();
      for (int p = 0; p < W; ++p) st_release_sys(reinterpret_cast<int*>(g.peer_comb_flag[p]) + g.rank, g.epoch);
      *g.done_ctr = 0;
    }
  }
}

// ------------------------------------------------------------------------------ combine
__global__ void __launch_bounds__(256) moe_combine_kernel(const __nv_bfloat16* __restrict__ comb,
                                                          __nv_bfloat16* __restrict__ out, const int* comb_flag,
                                                          int world, int epoch, int T, int K, int H,
                                                          volatile int* err, unsigned long long wait_ns) {
  __shared__ int s_ok;
  if (!cta_wait_all(comb_flag, world, epoch, err, 51, &s_ok, wait_ns)) return;
  const long long n8 = (long long)T * H / 8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const long long t = (i * 8) / H, c = (i * 8) % H;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < K; ++k) {
      const uint4 v = *reinterpret_cast<const uint4*>(comb + (t * K + k) * H + c);
      acc[0] += bf16_lo(v.x); acc[1] += bf16_hi(v.x); acc[2] += bf16_lo(v.y); acc[3] += bf16_hi(v.y);
      acc[4] += bf16_lo(v.z); acc[5] += bf16_hi(v.z); acc[6] += bf16_lo(v.w); acc[7] += bf16_hi(v.w);
    }
    *reinterpret_cast<uint4*>(out + t * H + c) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                   pack_bf16x2(acc[6], acc[7]));
  }
}

void make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && (cols * 2) % 16 == 0, "moe: TMA alignment");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {BK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult rc = cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                                             strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(rc == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(rc));
}

int sm_count(int dev) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace moe

// bufs (int64 CUDA tensor, per-peer addresses, [world] each): cnt_all, cnt_flag, recv_x,
// recv_meta, recv_w, arr_flag -- stacked as [6, world].
void moe_dispatch(torch::Tensor x, torch::Tensor topk_idx, torch::Tensor topk_w, int64_t E_l, int64_t rank,
                  int64_t world, int64_t epoch, int64_t cap_rows, torch::Tensor pair_pos, torch::Tensor gcount,
                  torch::Tensor grid_bar, torch::Tensor peers, torch::Tensor cnt_all, torch::Tensor cnt_flag,
                  torch::Tensor err) {
  using namespace moe;
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "moe_dispatch: x bf16 [T, H]");
  TORCH_CHECK(topk_idx.scalar_type() == torch::kInt32 && topk_w.scalar_type() == torch::kFloat32 &&
                  topk_idx.is_contiguous() && topk_w.is_contiguous(),
              "moe_dispatch: topk_idx int32 / topk_w float32 [T, K]");
  TORCH_CHECK(world <= MAXW && E_l <= MAXE && x.size(1) % 8 == 0, "moe_dispatch: limits");
  TORCH_CHECK(peers.scalar_type() == torch::kInt64 && peers.numel() >= 6 * world, "moe_dispatch: peer table");
  DispatchArgs a{};
  a.x = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr());
  a.topk_idx = topk_idx.data_ptr<int>();
  a.topk_w = topk_w.data_ptr<float>();
  a.T = x.size(0);
  a.K = topk_idx.size(1);
  a.H = x.size(1);
  a.E_l = E_l;
  a.rank = rank;
  a.world = world;
  a.epoch = epoch;
  a.cap_rows = cap_rows;
  TORCH_CHECK(pair_pos.numel() >= (int64_t)a.T * a.K, "moe_dispatch: pair_pos too small");
  a.pair_pos = pair_pos.data_ptr<int>();
  a.gcount = gcount.data_ptr<int>();
  a.grid_bar = grid_bar.data_ptr<int>();
  const int64_t* pt = peers.data_ptr<int64_t>();
  a.peer_cnt_all = pt;
  a.peer_cnt_flag = pt + world;
  a.peer_recv_x = pt + 2 * world;
  a.peer_recv_meta = pt + 3 * world;
  a.peer_recv_w = pt + 4 * world;
  a.peer_arr_flag = pt + 5 * world;
  a.cnt_all = cnt_all.data_ptr<int>();
  a.cnt_flag = cnt_flag.data_ptr<int>();
  a.err = err.data_ptr<int>();
  a.wait_ns = peer_wait_ns();
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_dispatch_kernel, 256, 0);
  // one warp per (token, k) pair, 8 per CTA; a small batch (decode) gets a small grid so
  // the grid barrier stays cheap
  const int want = static_cast<int>((static_cast<int64_t>(a.T) * a.K + 7) / 8);
  const int grid = std::max(1, std::min({sm_count(x.device().index()) * std::max(1, per_sm), 4 * 148, want}));
  void* args[] = {&a};
  AXR_CHECK_CUDA(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(moe_dispatch_kernel), dim3(grid), dim3(256),
                                             args, 0, at::cuda::getCurrentCUDAStream()));
}

// mode 0: a = recv_x [cap_rows, K], w = [E_l * N, K] (gate/up interleaved per 128 rows),
//         out = h [cap_rows, N/2]. mode 1: a = h [cap_rows, K], w = [E_l * N, K],
//         combine rows go to the origins' comb buffers.
void moe_gemm(torch::Tensor a, torch::Tensor w, int64_t mode, int64_t E_l, int64_t rank, int64_t world,
              int64_t epoch, torch::Tensor cnt_all, torch::Tensor cnt_flag, torch::Tensor arr_flag,
              c10::optional<torch::Tensor> h, c10::optional<torch::Tensor> recv_meta,
              c10::optional<torch::Tensor> recv_w, c10::optional<torch::Tensor> peer_comb,
              c10::optional<torch::Tensor> peer_comb_flag, torch::Tensor done_ctr, torch::Tensor err) {
  using namespace moe;
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == torch::kBFloat16 && a.is_contiguous(), "moe_gemm: a bf16");
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kBFloat16 && w.is_contiguous() && w.dim() == 2,
              "moe_gemm: w bf16 [E_l * N, K]");
  const int K = a.size(1);
  TORCH_CHECK(w.size(1) == K && w.size(0) % E_l == 0, "moe_gemm: shapes");
  const int N = w.size(0) / E_l;
  TORCH_CHECK(N % BN == 0 && K % BK == 0, "moe_gemm: N must be a multiple of 256, K of 64");
  TORCH_CHECK(world <= MAXW && E_l <= MAXE, "moe_gemm: limits");
  GemmArgs g{};
  g.mode = mode;
  g.rank = rank;
  g.world = world;
  g.E_l = E_l;
  g.N = N;
  g.K = K;
  g.epoch = epoch;
  g.cap_rows = a.size(0);
  g.cnt_all = cnt_all.data_ptr<int>();
  g.cnt_flag = cnt_flag.data_ptr<int>();
  g.arr_flag = arr_flag.data_ptr<int>();
  g.done_ctr = done_ctr.data_ptr<int>();
  g.err = err.data_ptr<int>();
  g.wait_ns = peer_wait_ns();
  if (mode == 0) {
    TORCH_CHECK(h.has_value() && h->size(0) >= a.size(0) && h->size(1) == N / 2 && h->stride(1) == 1,
                "moe_gemm: h [cap_rows, N/2]");
    g.h = reinterpret_cast<__nv_bfloat16*>(h->data_ptr());
    g.ldh = h->stride(0);
  } else {
    TORCH_CHECK(recv_meta.has_value() && recv_w.has_value() && peer_comb.has_value() && peer_comb_flag.has_value(),
                "moe_gemm: down mode needs recv_meta, recv_w, peer_comb, peer_comb_flag");
    g.recv_meta = reinterpret_cast<const int2*>(recv_meta->data_ptr<int>());
    g.recv_w = recv_w->data_ptr<float>();
    g.peer_comb = peer_comb->data_ptr<int64_t>();
    g.peer_comb_flag = peer_comb_flag->data_ptr<int64_t>();
  }
  CUtensorMap ta, tb;
  make_map(&ta, a.data_ptr(), a.size(0), K, BM);
  make_map(&tb, w.data_ptr(), w.size(0), K, BN);
  static bool attr = false;
  if (!attr) {
    AXR_CHECK_CUDA(cudaFuncSetAttribute(moe_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
    attr = true;
  }
  const int grid = sm_count(a.device().index());
  moe_gemm_kernel<<<grid, THREADS, SMEM, at::cuda::getCurrentCUDAStream()>>>(ta, tb, g);
  AXR_CHECK_CUDA(cudaGetLastError());
}

void moe_combine(torch::Tensor comb, torch::Tensor out, torch::Tensor comb_flag, int64_t world, int64_t epoch,
                 int64_t K, torch::Tensor err) {
  using namespace moe;
  const int T = out.size(0), H = out.size(1);
  TORCH_CHECK(out.is_contiguous() && out.scalar_type() == torch::kBFloat16 && H % 8 == 0, "moe_combine: out");
  TORCH_CHECK(comb.numel() >= (int64_t)T * K * H, "moe_combine: comb too small");
  const int grid = std::max(1, std::min(sm_count(out.device().index()) * 4,
                                        static_cast<int>(((int64_t)T * H / 8 + 255) / 256)));
  moe_combine_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(comb.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()),
      comb_flag.data_ptr<int>(), world, epoch, T, K, H, err.data_ptr<int>(), peer_wait_ns());
  AXR_CHECK_CUDA(cudaGetLastError());
}

}  // namespace axr
