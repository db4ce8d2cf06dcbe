// Dense projections of the single-GPU / data-parallel models on tcgen05, with the
// element-wise step that follows each projection fused into its epilogue.
//
//   out = epilogue(X W^T), X [M, K] bf16 activations, W [N, K] bf16 weights ("out x in"),
//   fp32 accumulation in tensor memory.
//
// Two kernels, chosen by the number of token rows M:
//
// * gemm_stream_kernel (M <= 256: decode steps, AMF-hit suffix prefills). The weights
//   are the only large operand, so the kernel is a weight stream: the MMA's M side is
//   128 weight rows (swap-AB), its N side the M token rows padded to NT (16..256).
//   The reduction is split over `splits` (<= 8) CTAs per 128-row tile so that every SM
//   keeps TMA loads of weights in flight. The CTAs of a tile form a thread-block cluster:
//   each parks its fp32 partial in its own shared memory and each sums a share of the
//   tile's token columns over all of them through distributed shared memory (in split
//   order, so the result does not depend on timing) and runs that share's epilogue; no
//   partial goes through global memory. The kernel is launched with
//   programmatic dependent launch: it lets the next kernel be scheduled as soon as its
//   own set-up is done, and it fills its TMA ring with weight tiles before it waits for
//   the previous kernel (griddepcontrol.wait), so the stream starts while the previous
//   kernel drains; activations and every epilogue input are read after the wait.
// * gemm_big_kernel (M > 256: prefills). Persistent, one CTA per SM, 128 x 256 output
//   tiles in a grouped raster, a 4-stage TMA ring, two 256-column TMEM accumulators so
//   the epilogue of tile i overlaps the MMAs of tile i + 1.
//
// Epilogues (both kernels):
//   STORE  : out = acc
//   RESID  : out = res + acc (res may be out itself: the residual stream updated in place)
//   SWIGLU : W rows are gate/up interleaved in groups of 64 (rows 128j..128j+63 = gate
//            features 64j.., rows 128j+64.. = up features 64j..); out[:, f] = silu(g) * u
//   ROPE   : W = [q heads | k heads | v heads] x 128 dims; rotate-half RoPE on q and k at
//            pos[m], q written to out, k and v stored at slots[m] of a bf16 paged cache
//            (slot < 0: not stored).
//
// Every wait is bounded (tc::mbar_wait: records a code in err and winds down). Every
// TMA load is a plain per-CTA load of this GPU's memory (no multicast).
// Reference counterpart: the dense projections the reference leaves to vLLM / llama.cpp
// library GEMMs (axropus/server.py:110, core/engine.cpp llama_decode).
#include <algorithm>
#include <cstdlib>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm_dense.h"
#include "tc_common.cuh"

namespace axr {
namespace dense {

struct EpiArgs {
  __nv_bfloat16* out;
  long long ldo;
  const __nv_bfloat16* res;  // RESID
  long long ldr;
  const int* pos;             // ROPE
  const int* slots;
  const float* cos_sin;       // [n_pos, 128]: cos [0, 64), sin [64, 128)
  int n_pos;
  char* kc;                   // bf16 paged cache of this layer: unit (blk, head) at blk*blk_stride + head*head_stride
  char* vc;
  long long blk_stride, head_stride;
  int Hq, Hkv;
};

struct Args {
  int M, N, K;
  int splits;   // stream kernel: CTAs per 128-row weight tile
  unsigned long long* trace;  // stream kernel timeline (AXR_DENSE_TRACE=1): 8 %globaltimer stamps per CTA
  volatile int* err;
  EpiArgs e;
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float silu(float g) { return g / (1.f + __expf(-g)); }

__device__ __forceinline__ char* align1024(char* p) {
  return reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Where row m of k/v head h goes in the paged cache (nullptr: not stored).
__device__ __forceinline__ __nv_bfloat16* cache_row(const EpiArgs& e, bool is_v, int h, int m) {
  const int slot = e.slots[m];
  if (slot < 0) return nullptr;
  char* unit = (is_v ? e.vc : e.kc) + (long long)(slot / kPage) * e.blk_stride + (long long)h * e.head_stride;
  return reinterpret_cast<__nv_bfloat16*>(unit + (long long)(slot % kPage) * 128 * 2);
}

// =====================================================================================
// weight-streaming kernel
// =====================================================================================
template <int NT>
struct StreamCfg {
  static constexpr int ST = NT <= 16 ? 6 : NT <= 32 ? 5 : NT <= 64 ? 4 : NT <= 128 ? 3 : 4;
  static constexpr int A_BYTES = 128 * 64 * 2;  // 128 weight rows x 64 k
  static constexpr int B_BYTES = NT * 64 * 2;   // NT token rows x 64 k
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int SMEM = 1024 + ST * STAGE + 128;
  static constexpr int TMEM_COLS = NT < 32 ? 32 : NT;
  static constexpr int CH = NT < 32 ? NT : 32;  // epilogue columns (tokens) per TMEM load
  static constexpr int CTAS_PER_SM = NT <= 128 ? 2 : 1;
};

// Every thread of every CTA of the cluster (release / acquire: shared-memory writes before
// it are visible to the cluster after it).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The float at this CTA's shared address `p`, read from cluster CTA `rank`'s shared memory.
__device__ __forceinline__ float ld_dsmem(const float* p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(tc::smem_u32(p)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

template <int CH>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, float (&v)[CH]) {
  if constexpr (CH == 16) {
    uint32_t r[16];
    tc::tmem_ld16(taddr, r);
    tc::tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
  } else {
    uint32_t r[32];
    tc::tmem_ld32(taddr, r);
    tc::tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  }
}

// Epilogue of one chunk of CH token columns. Thread t holds weight row r = t of the tile
// (feature n0 + r) for tokens c0 .. c0 + CH - 1. sx: [128][CH + 1] fp32 exchange space.
// Every global input of a chunk is loaded before the chunk's first store: `out` may be
// `res` (the residual stream updated in place), so a load after a store could not be
// issued early and each token would cost a full memory round trip.
template <int EPI, int CH>
__device__ __forceinline__ void stream_epilogue(const Args& g, int tile, int c0, const float (&v)[CH], float* sx) {
  const int r = threadIdx.x;
  const EpiArgs& e = g.e;
  if constexpr (EPI == kStore || EPI == kResid) {
    const int n = tile * 128 + r;
    if (n >= g.N) return;
    float rv[CH];
#pragma unroll
    for (int j = 0; j < CH; ++j) {
      rv[j] = 0.f;
      if constexpr (EPI == kResid) {
        if (c0 + j < g.M) rv[j] = __bfloat162float(e.res[(long long)(c0 + j) * e.ldr + n]);
      }
    }
#pragma unroll
    for (int j = 0; j < CH; ++j)
      if (c0 + j < g.M) e.out[(long long)(c0 + j) * e.ldo + n] = __float2bfloat16(v[j] + rv[j]);
  } else {
#pragma unroll
    for (int j = 0; j < CH; ++j) sx[r * (CH + 1) + j] = v[j];
    __syncthreads();
    const int d = r & 63, jj = r >> 6;
    constexpr int JN = CH / 2;  // tokens of this thread: jj, jj + 2, ...
    if constexpr (EPI == kSwiGLU) {
      const int f = tile * 64 + d;
#pragma unroll
      for (int t = 0; t < JN; ++t) {
        const int j = jj + 2 * t, m = c0 + j;
        if (m < g.M) {
          const float gt = sx[d * (CH + 1) + j], up = sx[(d + 64) * (CH + 1) + j];
          e.out[(long long)m * e.ldo + f] = __float2bfloat16(silu(gt) * up);
        }
      }
    } else {  // ROPE: tile = head row hr of [q | k | v]
      const int hr = tile;
      const bool rot = hr < e.Hq + e.Hkv, is_q = hr < e.Hq, is_v = !rot;
      float co[JN], si[JN];
      __nv_bfloat16* dst[JN];
#pragma unroll
      for (int t = 0; t < JN; ++t) {  // positions, slots, cos / sin first
        const int m = c0 + jj + 2 * t;
        co[t] = 1.f;
        si[t] = 0.f;
        dst[t] = nullptr;
        if (m < g.M) {
          if (rot) {
            const int ps = min(max(e.pos[m], 0), e.n_pos - 1);
            co[t] = e.cos_sin[(long long)ps * 128 + d];
            si[t] = e.cos_sin[(long long)ps * 128 + 64 + d];
          }
          dst[t] = is_q ? e.out + (long long)m * e.ldo + hr * 128
                        : cache_row(e, is_v, is_v ? hr - e.Hq - e.Hkv : hr - e.Hq, m);
        }
      }
#pragma unroll
      for (int t = 0; t < JN; ++t) {
        if (dst[t] == nullptr) continue;
        const int j = jj + 2 * t;
        const float x1 = sx[d * (CH + 1) + j], x2 = sx[(d + 64) * (CH + 1) + j];
        dst[t][d] = __float2bfloat16(x1 * co[t] - x2 * si[t]);
        dst[t][d + 64] = __float2bfloat16(x2 * co[t] + x1 * si[t]);
      }
    }
    __syncthreads();
  }
}

template <int NT, int EPI>
__global__ void __launch_bounds__(128) gemm_stream_kernel(const __grid_constant__ CUtensorMap tmW,
                                                          const __grid_constant__ CUtensorMap tmX, Args g) {
  using C = StreamCfg<NT>;
  extern __shared__ __align__(1024) char smem_raw[];
  char* base = align1024(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(base + C::ST * C::STAGE);
  uint64_t* empty = full + C::ST;
  uint64_t* accb = empty + C::ST;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accb + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * 128;
  const int nk = (g.K + 63) / 64;
  const int kb0 = static_cast<int>((long long)split * nk / g.splits);
  const int kb1 = static_cast<int>((long long)(split + 1) * nk / g.splits);
  const int nkb = kb1 - kb0;
  unsigned long long* tr = g.trace ? g.trace + 8ull * (blockIdx.y * gridDim.x + blockIdx.x) : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = tc::globaltimer();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::ST; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(accb, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmW);
    tc::prefetch_tmap(&tmX);
  }
  if (warp == 2) {
    tc::tmem_alloc(tmem_slot, C::TMEM_COLS);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tr && threadIdx.x == 0) tr[1] = tc::globaltimer();
  // Set-up done (tensor memory held): the next kernel may come up on free SM space and
  // start its own independent loads while this one streams.
  if (threadIdx.x == 0) griddep_launch();

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer: weights first (independent of earlier kernels), then activations
    const int pre = min(C::ST, nkb);
    for (int i = 0; i < pre; ++i) {
      tc::mbar_arrive_expect_tx(&full[i], C::STAGE);
      tc::tma_load_2d(base + i * C::STAGE, &tmW, (kb0 + i) * 64, n0, &full[i]);
    }
    griddep_wait();
    for (int i = 0; i < pre; ++i) tc::tma_load_2d(base + i * C::STAGE + C::A_BYTES, &tmX, (kb0 + i) * 64, 0, &full[i]);
    int issued = pre;
    bool ok = true;
    for (int i = pre; i < nkb; ++i) {
      const int s = i % C::ST;
      if (!tc::mbar_wait(&empty[s], ((i / C::ST) + 1) & 1, g.err, 1)) { ok = false; break; }
      tc::mbar_arrive_expect_tx(&full[s], C::STAGE);
      tc::tma_load_2d(base + s * C::STAGE, &tmW, (kb0 + i) * 64, n0, &full[s]);
      tc::tma_load_2d(base + s * C::STAGE + C::A_BYTES, &tmX, (kb0 + i) * 64, 0, &full[s]);
      issued = i + 1;
    }
    if (!ok) {  // let this thread's loads land before the CTA can exit
      for (int i = max(0, issued - C::ST); i < issued; ++i) tc::mbar_wait_quiet(&full[i % C::ST], (i / C::ST) & 1);
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = tc::idesc_bf16_f32(128, NT);
    bool ok = true;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % C::ST;
      if (!tc::mbar_wait(&full[s], (i / C::ST) & 1, g.err, 2)) { ok = false; break; }
      if (tr && (i == 0 || i == nkb - 1)) tr[i == 0 ? 2 : 3] = tc::globaltimer();
      tc::tc_fence_after();
      const uint32_t a_addr = tc::smem_u32(base + s * C::STAGE);
      const uint32_t b_addr = a_addr + C::A_BYTES;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        tc::mma_f16_ss(tmem, tc::smem_desc_k_sw128(a_addr + kk * 32), tc::smem_desc_k_sw128(b_addr + kk * 32), idesc,
                       (i | kk) != 0);
      tc::mma_commit(&empty[s]);
    }
    tc::mma_commit(accb);
    if (!ok) tc::mbar_wait_quiet(accb, 0);
  }
  __syncwarp();

  // ---------------- epilogue (all 4 warps; warp w reads TMEM lanes 32w..32w+31)
  bool ready = tc::mbar_wait(accb, 0, g.err, 3);
  if (tr && threadIdx.x == 0) tr[4] = tc::globaltimer();
  tc::tc_fence_after();
  griddep_wait();  // residual, positions and slots come from earlier kernels
  ready = __syncthreads_and(ready && *g.err == 0) != 0;
  const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const int r = threadIdx.x;
  const int mt = min(g.M, NT);  // token columns that hold rows
  if (g.splits == 1) {
    float* sx = reinterpret_cast<float*>(base);  // the TMA ring is idle once the accumulator is complete
    if (ready) {
#pragma unroll 1
      for (int c0 = 0; c0 < mt; c0 += C::CH) {
        float v[C::CH];
        tmem_ld_chunk<C::CH>(trow + c0, v);
        stream_epilogue<EPI, C::CH>(g, tile, c0, v, sx);
      }
    }
  } else {
    // split-K inside the cluster: each CTA parks its fp32 partial [NT][128] in its idle
    // ring, and after a cluster barrier CTA `split` sums the CHR-token chunks c with
    // c % splits == split over every CTA's shared memory (distributed shared memory, in
    // split order: deterministic) and runs their epilogue; a second barrier keeps every
    // partial alive until all CTAs have read it. Both barriers are reached by every
    // thread of every CTA, failed or not. Chunks are small enough that every CTA of the
    // cluster takes a share (32 tokens over 8 CTAs: 4 each), and each thread issues its
    // loads from all splits before the first add (one remote round trip, not one per
    // split): the reduction tail was 4-5 us of a 13-16 us projection with 16-token chunks
    // summed split by split.
    constexpr int CHR = NT <= 32 ? 4 : (NT <= 64 ? 8 : 16);
    constexpr int QB = CHR <= 4 ? 8 : (CHR <= 8 ? 4 : 2);  // splits per batch of loads
    float* part = reinterpret_cast<float*>(base);
    float* sx = part + NT * 128;
    if (ready) {
#pragma unroll 1
      for (int c0 = 0; c0 < mt; c0 += C::CH) {
        float v[C::CH];
        tmem_ld_chunk<C::CH>(trow + c0, v);
#pragma unroll
        for (int j = 0; j < C::CH; ++j) part[(c0 + j) * 128 + r] = v[j];
      }
    }
    cluster_sync();
    if (tr && threadIdx.x == 0) tr[5] = tc::globaltimer();
    if (ready) {
      const int n = tile * 128 + r;
#pragma unroll 1
      for (int c0 = split * CHR; c0 < mt; c0 += g.splits * CHR) {
        float v[CHR], rv[CHR];
#pragma unroll
        for (int j = 0; j < CHR; ++j) {
          v[j] = 0.f;
          rv[j] = 0.f;
          if constexpr (EPI == kResid) {  // epilogue input loaded with the partials
            if (n < g.N && c0 + j < g.M) rv[j] = __bfloat162float(g.e.res[(long long)(c0 + j) * g.e.ldr + n]);
          }
        }
#pragma unroll 1
        for (int q0 = 0; q0 < g.splits; q0 += QB) {
          float pv[QB][CHR];
#pragma unroll
          for (int qq = 0; qq < QB; ++qq)
#pragma unroll
            for (int j = 0; j < CHR; ++j)
              pv[qq][j] = q0 + qq < g.splits ? ld_dsmem(part + (c0 + j) * 128 + r, q0 + qq) : 0.f;
#pragma unroll
          for (int qq = 0; qq < QB; ++qq)
#pragma unroll
            for (int j = 0; j < CHR; ++j) v[j] += pv[qq][j];
        }
        if constexpr (EPI == kStore || EPI == kResid) {
          if (n < g.N) {
#pragma unroll
            for (int j = 0; j < CHR; ++j)
              if (c0 + j < g.M) g.e.out[(long long)(c0 + j) * g.e.ldo + n] = __float2bfloat16(v[j] + rv[j]);
          }
        } else {
          stream_epilogue<EPI, CHR>(g, tile, c0, v, sx);
        }
      }
    }
    if (tr && threadIdx.x == 0) tr[6] = tc::globaltimer();
    cluster_sync();
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 2) tc::tmem_dealloc(tmem, C::TMEM_COLS);
  if (tr && threadIdx.x == 0) tr[7] = tc::globaltimer();
}

// =====================================================================================
// persistent big-M kernel
// =====================================================================================
constexpr int BM = 128, BN = 256, BK = 64, BST = 4;
constexpr int BA_BYTES = BM * BK * 2, BB_BYTES = BN * BK * 2;
constexpr int BSMEM = 1024 + BST * (BA_BYTES + BB_BYTES) + 256;
constexpr int BTHREADS = 192;
constexpr int BGROUP_M = 16;

__device__ __forceinline__ void big_tile(int t, int num_m, int num_n, int& mt, int& nt) {
  const int group = BGROUP_M * num_n;
  const int first = (t / group) * BGROUP_M;
  const int gm = min(num_m - first, BGROUP_M);
  const int in = t - (t / group) * group;
  mt = first + in % gm;
  nt = in / gm;
}

__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tc::tmem_ld32(taddr, r);
  tc::tmem_ld_wait();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// 32 floats -> 32 bf16 at dst (16-byte aligned), or element-wise up to `n` valid columns.
__device__ __forceinline__ void store32(__nv_bfloat16* dst, const float (&v)[32], int n) {
  if (n >= 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
      reinterpret_cast<uint4*>(dst)[q] =
          make_uint4(pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]), pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]),
                     pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]), pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n) dst[j] = __float2bfloat16(v[j]);
  }
}

// Epilogue of one tile: thread = token row m, TMEM columns = features of the tile.
template <int EPI>
__device__ __forceinline__ void big_epilogue(const Args& g, uint32_t tacc, int m, int mt, int nt) {
  const EpiArgs& e = g.e;
  const bool row_ok = m < g.M;
  if constexpr (EPI == kStore || EPI == kResid) {
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32f(tacc + c, v);
      const int n = nt * BN + c;
      if (!row_ok || n >= g.N) continue;
      if constexpr (EPI == kResid) {
        const __nv_bfloat16* rp = e.res + (long long)m * e.ldr + n;
        if (n + 32 <= g.N && (reinterpret_cast<uintptr_t>(rp) & 15) == 0) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 x = reinterpret_cast<const uint4*>(rp)[q];
            v[q * 8 + 0] += bf16_lo(x.x); v[q * 8 + 1] += bf16_hi(x.x);
            v[q * 8 + 2] += bf16_lo(x.y); v[q * 8 + 3] += bf16_hi(x.y);
            v[q * 8 + 4] += bf16_lo(x.z); v[q * 8 + 5] += bf16_hi(x.z);
            v[q * 8 + 6] += bf16_lo(x.w); v[q * 8 + 7] += bf16_hi(x.w);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (n + j < g.N) v[j] += __bfloat162float(rp[j]);
        }
      }
      store32(e.out + (long long)m * e.ldo + n, v, g.N - n);
    }
  } else if constexpr (EPI == kSwiGLU) {
    // 256 columns = 2 gate/up pairs of 64 -> 128 outputs
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
#pragma unroll 1
      for (int p = 0; p < 64; p += 32) {
        float gt[32], up[32];
        tmem_ld32f(tacc + q * 128 + p, gt);
        tmem_ld32f(tacc + q * 128 + 64 + p, up);
        const int f = nt * 128 + q * 64 + p;
        if (!row_ok || 2 * f >= g.N) continue;
#pragma unroll
        for (int j = 0; j < 32; ++j) gt[j] = silu(gt[j]) * up[j];
        store32(e.out + (long long)m * e.ldo + f, gt, g.N / 2 - f);
      }
    }
  } else {  // ROPE: 256 columns = head rows 2nt, 2nt+1
    const int ps = row_ok ? min(max(e.pos[m], 0), e.n_pos - 1) : 0;
    const float* cs = e.cos_sin + (long long)ps * 128;
#pragma unroll 1
    for (int q = 0; q < 2; ++q) {
      const int hr = nt * 2 + q;
      const bool rot = hr < e.Hq + e.Hkv, is_q = hr < e.Hq, is_v = !rot;
      __nv_bfloat16* dst = nullptr;
      if (row_ok && hr < e.Hq + 2 * e.Hkv) {
        dst = is_q ? e.out + (long long)m * e.ldo + hr * 128
                   : cache_row(e, is_v, is_v ? hr - e.Hq - e.Hkv : hr - e.Hq, m);
      }
#pragma unroll 1
      for (int p = 0; p < 64; p += 32) {
        float x1[32], x2[32];
        tmem_ld32f(tacc + q * 128 + p, x1);
        tmem_ld32f(tacc + q * 128 + 64 + p, x2);
        if (dst == nullptr) continue;
        if (rot) {
#pragma unroll
          for (int j4 = 0; j4 < 32; j4 += 4) {
            const float4 co = *reinterpret_cast<const float4*>(cs + p + j4);
            const float4 si = *reinterpret_cast<const float4*>(cs + 64 + p + j4);
            const float c4[4] = {co.x, co.y, co.z, co.w}, s4[4] = {si.x, si.y, si.z, si.w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float a = x1[j4 + u], b = x2[j4 + u];
              x1[j4 + u] = a * c4[u] - b * s4[u];
              x2[j4 + u] = b * c4[u] + a * s4[u];
            }
          }
        }
        store32(dst + p, x1, 32);
        store32(dst + 64 + p, x2, 32);
      }
    }
  }
}

// Roles: warp 0 TMA producer, warp 1 MMA issuer, warps 2..5 epilogue (TMEM lane group
// warp % 4), warp 2 also owns the 512 TMEM columns.
template <int EPI>
__global__ void __launch_bounds__(BTHREADS, 1) gemm_big_kernel(const __grid_constant__ CUtensorMap tmX,
                                                               const __grid_constant__ CUtensorMap tmW, Args g) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* base = align1024(smem_raw);
  char* sA = base;
  char* sB = base + BST * BA_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + BST * BB_BYTES);
  uint64_t* empty = full + BST;
  uint64_t* accf = empty + BST;  // [2]
  uint64_t* acce = accf + 2;     // [2]
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (g.M + BM - 1) / BM, num_n = (g.N + BN - 1) / BN;
  const int tiles = num_m * num_n;
  const int nk = (g.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < BST; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&accf[b], 1);
      tc::mbar_init(&acce[b], 4);
    }
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmX);
    tc::prefetch_tmap(&tmW);
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
      bool waited = false;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        int mt, nt;
        big_tile(t, num_m, num_n, mt, nt);
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % BST;
          if (it >= BST && !tc::mbar_wait(&empty[s], ((it / BST) + 1) & 1, g.err, 1)) { ok = false; break; }
          tc::mbar_arrive_expect_tx(&full[s], BA_BYTES + BB_BYTES);
          tc::tma_load_2d(sB + s * BB_BYTES, &tmW, kt * BK, nt * BN, &full[s]);  // weights: no dependency
          if (!waited) {
            griddep_wait();
            waited = true;
          }
          tc::tma_load_2d(sA + s * BA_BYTES, &tmX, kt * BK, mt * BM, &full[s]);
        }
      }
      if (!waited) griddep_wait();
      if (!ok) {
        for (int j = max(0, it - BST); j < it; ++j) tc::mbar_wait_quiet(&full[j % BST], (j / BST) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN);
      int it = 0, i = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
        const int buf = i & 1;
        if (i >= 2 && !tc::mbar_wait(&acce[buf], ((i >> 1) + 1) & 1, g.err, 6)) break;
        tc::tc_fence_after();
        bool ok = true;
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % BST;
          if (!tc::mbar_wait(&full[s], (it / BST) & 1, g.err, 2)) { ok = false; break; }
          tc::tc_fence_after();
          const uint32_t a_addr = tc::smem_u32(sA + s * BA_BYTES), b_addr = tc::smem_u32(sB + s * BB_BYTES);
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
    griddep_wait();  // residual / positions / slots come from earlier kernels
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      int mt, nt;
      big_tile(t, num_m, num_n, mt, nt);
      const int buf = i & 1;
      bool ok = tc::mbar_wait(&accf[buf], (i >> 1) & 1, g.err, 3);
      ok = __all_sync(0xffffffffu, ok) && __shfl_sync(0xffffffffu, *g.err, 0) == 0;
      tc::tc_fence_after();
      if (!ok) break;
      const int m = mt * BM + lg * 32 + lane;
      big_epilogue<EPI>(g, tmem + buf * BN + (static_cast<uint32_t>(lg * 32) << 16), m, mt, nt);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acce[buf]);
    }
  }
  // The next kernel is released only once this CTA's tiles are done: a compute-bound
  // prefill GEMM gains nothing from company, and CTAs of the next kernel parked in their
  // wait beside it cost clock under the power cap (measured: an 8320-token forward
  // 127 ms with the release here or no early launch at all, 136 ms releasing at the start).
  if (threadIdx.x == 0) griddep_launch();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 2) tc::tmem_dealloc(tmem, 512);
}

// =====================================================================================
// persistent CTA-pair kernel (tcgen05 cta_group::2): one 256 x 256 output tile per pair
// =====================================================================================
// The two CTAs of a cluster run the tensor cores of two SMs as one 256-row MMA: CTA r
// loads rows [128 r, 128 r + 128) of the tile's X rows and of its W rows (half of B
// each) into its own shared memory; the leader (r = 0) issues tcgen05.mma.cta_group::2
// with M = N = 256, which reads A and B from both CTAs' shared memory and accumulates
// each CTA's 128 rows x 256 columns in that CTA's TMEM. Per SM that is 32 KB of operands
// per 64-deep k step instead of 48 KB for a 1-CTA 128 x 256 tile at the same MMA rate:
// a third less L2 -> SM and shared-memory traffic (and energy under the power cap) per
// FLOP (8320 x 28672 x 4096 + SwiGLU: 1.261 ms against 1.333 ms for the 1-CTA kernel).
//
// Synchronisation: both CTAs' TMA loads (plain per-CTA loads of this GPU's memory, no
// multicast; the .cta_group::2 form lets a load complete on the peer's barrier) count
// their bytes on the leader's full[s], for which the leader's producer expects both
// halves. The leader's commits are multicast to both CTAs (stage free: empty[s];
// accumulator ready: accf[b]); both CTAs' epilogue warps arrive on the leader's acce[b]
// (count 8) when their half of a TMEM buffer is drained. A cluster barrier at the end
// keeps either CTA from leaving while the other may still read its shared memory or
// arrive on its barriers. (Measured and dropped: each CTA's loads completing on its own
// barrier and a peer thread relaying the completion to the leader -- the extra hop
// starved the 6-stage ring and halved the rate.)
constexpr int PST = 6;
constexpr int PA_BYTES = 128 * BK * 2;   // this CTA's 128 X rows
constexpr int PB_BYTES = 128 * BK * 2;   // this CTA's 128 W rows (half of the tile's 256)
constexpr int PSTAGE = PA_BYTES + PB_BYTES;
constexpr int PSMEM = 1024 + PST * PSTAGE + 256;
constexpr int PBM = 256, PBN = 256;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_rank(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(tc::smem_u32(p)), "r"(rank));
  return a;
}
// Arrive on the barrier at shared::cluster address `a` (possibly another CTA's), release
// at cluster scope: the arriving thread's earlier writes (and fenced tcgen05 reads) are
// ordered before the waiter's acquire.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t a) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(a) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(tc::smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded cluster-scope wait (barriers that a thread of the other CTA arrives on).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t phase, volatile int* err, int code) {
  if (mbar_try_wait_cluster(bar, phase)) return true;
  const unsigned long long t0 = tc::globaltimer();
  while (true) {
    if (mbar_try_wait_cluster(bar, phase)) return true;
    if (*err != 0) return false;
    if (tc::globaltimer() - t0 > tc::kWaitLimitNs) {
      atomicCAS(const_cast<int*>(err), 0, code);
      return false;
    }
  }
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_u32(dst)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::);
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void mma_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// Arrive on the barrier at this shared offset in both CTAs of the pair once every earlier
// MMA of this thread has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          tc::smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// 2D tiled TMA load into this CTA's shared memory whose completion is counted on the
// barrier at shared::cluster address `bar_cluster` (the pair leader's); no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(tc::smem_u32(smem)),
      "l"(map), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}

template <int EPI>
__global__ void __launch_bounds__(BTHREADS, 1) gemm_pair_kernel(const __grid_constant__ CUtensorMap tmX,
                                                                const __grid_constant__ CUtensorMap tmW, Args g) {
  extern __shared__ __align__(1024) char smem_raw[];
  char* base = align1024(smem_raw);  // same offset in both CTAs (same kernel, same layout)
  char* sA = base;
  char* sB = base + PST * PA_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + PST * PB_BYTES);
  uint64_t* empty = full + PST;
  uint64_t* accf = empty + PST;  // [2]
  uint64_t* acce = accf + 2;     // [2] (used in the leader)
  uint64_t* drain = acce + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int num_m = (g.M + PBM - 1) / PBM, num_n = (g.N + PBN - 1) / PBN;
  const int tiles = num_m * num_n;
  const int nk = (g.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < PST; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&accf[b], 1);
      tc::mbar_init(&acce[b], 8);
    }
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmX);
    tc::prefetch_tmap(&tmW);
  }
  if (warp == 2) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc::tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any remote arrive or multicast commit
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer (both CTAs): this CTA's halves
      int it = 0;
      bool ok = true, waited = false;
      for (int t = pair; ok && t < tiles; t += pairs) {
        int mt, nt;
        big_tile(t, num_m, num_n, mt, nt);
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = it % PST;
          if (it >= PST && !tc::mbar_wait(&empty[s], ((it / PST) + 1) & 1, g.err, 1)) { ok = false; break; }
          const int wy = nt * PBN + static_cast<int>(rank) * 128, xy = mt * PBM + static_cast<int>(rank) * 128;
          // both CTAs' bytes complete on the leader's full[s]; the leader expects them all
          if (rank == 0) tc::mbar_arrive_expect_tx(&full[s], 2 * PSTAGE);
          const uint32_t bar = mapa_rank(&full[s], 0);
          tma_load_2d_pair(sB + s * PB_BYTES, &tmW, kt * BK, wy, bar);
          if (!waited) {
            griddep_wait();
            waited = true;
          }
          tma_load_2d_pair(sA + s * PA_BYTES, &tmX, kt * BK, xy, bar);
        }
      }
      if (!waited) griddep_wait();
      if (!ok && rank == 0) {
        // let the pair's loads land before shared memory can be released: the leader's
        // barriers count both CTAs' bytes (the peer's in-flight loads land long before the
        // bounded waits of the failed roles run out and both CTAs reach the final barrier)
        for (int j = max(0, it - PST); j < it; ++j) tc::mbar_wait_quiet(&full[j % PST], (j / PST) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      if (rank == 0) {  // ---------------- MMA issuer for the pair
        constexpr uint32_t idesc = tc::idesc_bf16_f32(PBM, PBN);
        int it = 0, i = 0;
        for (int t = pair; t < tiles; t += pairs, ++i) {
          const int buf = i & 1;
          if (i >= 2 && !mbar_wait_cluster(&acce[buf], ((i >> 1) + 1) & 1, g.err, 6)) break;
          tc::tc_fence_after();
          bool ok = true;
          for (int kt = 0; kt < nk; ++kt, ++it) {
            const int s = it % PST;
            if (!mbar_wait_cluster(&full[s], (it / PST) & 1, g.err, 2)) { ok = false; break; }
            tc::tc_fence_after();
            const uint32_t a_addr = tc::smem_u32(sA + s * PA_BYTES), b_addr = tc::smem_u32(sB + s * PB_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
              mma_pair(tmem + buf * PBN, tc::smem_desc_k_sw128(a_addr + kk * 32),
                       tc::smem_desc_k_sw128(b_addr + kk * 32), idesc, (kt | kk) != 0);
            mma_commit_pair(&empty[s]);
          }
          mma_commit_pair(&accf[buf]);
          if (!ok) break;
        }
        mma_commit_pair(drain);  // fires in both CTAs once every MMA of the pair is done
      }
      tc::mbar_wait_quiet(drain, 0);  // no MMA still reads this CTA's shared memory / writes its TMEM
    }
  } else {
    // ---------------- epilogue warps 2..5 (both CTAs): this CTA's 128 rows of each tile
    const int lg = warp & 3;
    griddep_wait();  // residual / positions / slots come from earlier kernels
    const uint32_t acce_leader = mapa_rank(&acce[0], 0);
    int i = 0;
    for (int t = pair; t < tiles; t += pairs, ++i) {
      int mt, nt;
      big_tile(t, num_m, num_n, mt, nt);
      const int buf = i & 1;
      bool ok = tc::mbar_wait(&accf[buf], (i >> 1) & 1, g.err, 3);
      ok = __all_sync(0xffffffffu, ok) && __shfl_sync(0xffffffffu, *g.err, 0) == 0;
      tc::tc_fence_after();
      if (!ok) break;
      const int m = mt * PBM + static_cast<int>(rank) * 128 + lg * 32 + lane;
      big_epilogue<EPI>(g, tmem + buf * PBN + (static_cast<uint32_t>(lg * 32) << 16), m, mt, nt);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_leader + buf * 8);
    }
  }
  __syncwarp();
  if (threadIdx.x == 0) griddep_launch();
  tc::tc_fence_before();
  cluster_sync();  // neither CTA leaves while the other may read its shared memory or arrive on its barriers
  tc::tc_fence_after();
  if (warp == 2) tmem_dealloc_pair(tmem, 512);
}

// =====================================================================================
// host
// =====================================================================================
namespace {

bool make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count(int dev) {
  static int cached[64] = {0};
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (dev >= 0 && dev < 64) cached[dev] = sms;
  return sms;
}

// Programmatic dependent launch (AXR_DENSE_PDL=0 or AXR_PDL=0 turns it off, for measurements).
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("AXR_DENSE_PDL");
    return !(e && e[0] == '0') && pdl_enabled_env();
  }();
  return on;
}

// cluster_y > 1: clusters of (1, cluster_y, 1) CTAs (the split-K CTAs of one weight tile).
template <typename Kernel>
cudaError_t launch_dense(Kernel kernel, dim3 grid, dim3 block, int smem, cudaStream_t st, const CUtensorMap& m0,
                       const CUtensorMap& m1, const Args& g, int cluster_y = 1, int cluster_x = 1) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_y > 1 || cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = cluster_y;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, m0, m1, g);
}

template <int NT, int EPI>
cudaError_t launch_stream(const CUtensorMap& tw, const CUtensorMap& tx, const Args& g, cudaStream_t st) {
  using C = StreamCfg<NT>;
  auto kernel = gemm_stream_kernel<NT, EPI>;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  return launch_dense(kernel, dim3((g.N + 127) / 128, g.splits), dim3(128), C::SMEM, st, tw, tx, g, g.splits);
}

template <int EPI>
cudaError_t launch_stream_nt(int nt, const CUtensorMap& tw, const CUtensorMap& tx, const Args& g, cudaStream_t st) {
  switch (nt) {
    case 16: return launch_stream<16, EPI>(tw, tx, g, st);
    case 32: return launch_stream<32, EPI>(tw, tx, g, st);
    case 64: return launch_stream<64, EPI>(tw, tx, g, st);
    case 128: return launch_stream<128, EPI>(tw, tx, g, st);
    default: return launch_stream<256, EPI>(tw, tx, g, st);
  }
}

template <int EPI>
cudaError_t launch_big(const CUtensorMap& tx, const CUtensorMap& tw, const Args& g, int dev, cudaStream_t st) {
  auto kernel = gemm_big_kernel<EPI>;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BSMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int tiles = ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
  const int grid = std::max(1, std::min(tiles, sm_count(dev)));
  return launch_dense(kernel, dim3(grid), dim3(BTHREADS), BSMEM, st, tx, tw, g);
}

// AXR_DENSE_PAIR=0 runs prefill-sized GEMMs on the 1-CTA kernel (for measurements).
bool pair_enabled() {
  static const bool on = [] {
    const char* e = getenv("AXR_DENSE_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// Clusters of the pair kernel that fit the GPU at once (per device, cached): the
// persistent grid must be resident in one wave, and GPCs with an odd number of free SMs
// hold fewer pairs than SMs / 2.
template <int EPI>
int pair_clusters(int dev) {
  static const int forced = [] {
    const char* e = getenv("AXR_DENSE_PAIR_CLUSTERS");
    return e ? atoi(e) : 0;
  }();
  if (forced > 0) return forced;
  static int cached[64] = {0};
  if (dev >= 0 && dev < 64 && cached[dev]) return cached[dev];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74);
  cfg.blockDim = dim3(BTHREADS);
  cfg.dynamicSmemBytes = PSMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<EPI>, &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = sm_count(dev) / 2;
  }
  if (dev >= 0 && dev < 64) cached[dev] = n;
  return n;
}

template <int EPI>
cudaError_t launch_pair(const CUtensorMap& tx, const CUtensorMap& tw, const Args& g, int dev, cudaStream_t st) {
  auto kernel = gemm_pair_kernel<EPI>;
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PSMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int tiles = ((g.M + PBM - 1) / PBM) * ((g.N + PBN - 1) / PBN);
  const int clusters = std::max(1, std::min(tiles, pair_clusters<EPI>(dev)));
  return launch_dense(kernel, dim3(2 * clusters), dim3(BTHREADS), PSMEM, st, tx, tw, g, 1, 2);
}

}  // namespace

int pair_grid_clusters(int dev) {
  cudaFuncSetAttribute(gemm_pair_kernel<kStore>, cudaFuncAttributeMaxDynamicSharedMemorySize, PSMEM);
  return pair_clusters<kStore>(dev);
}

// Largest split count whose partials of one chunk (CH tokens) fit the TMA ring.
// Split-K CTAs of one weight tile form a cluster: at most the portable cluster size.
int stream_max_splits(int nt) {
  (void)nt;
  return 8;
}

int stream_nt(int64_t M) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  if (M <= 256) return 256;
  return 0;
}

// Enough CTAs to give every SM its resident share of weight tiles, each CTA keeping at
// least 4 k-blocks (256 of K).
// CTAs per weight tile: as many as fit (<= 8, the portable cluster size; >= 8 k-blocks
// each) while all tiles' clusters stay within ~7/8 of the resident CTA slots. Clusters
// are placed whole inside a GPC, so a grid that asks for every slot does not become
// resident at once, and its last clusters run as a second wave (measured: 288 CTAs of
// 6-CTA clusters took 1.6x the time of 240 CTAs of 5).
int stream_splits(int64_t M, int64_t N, int64_t K, int sms) {
  const int nt = stream_nt(M);
  const int64_t tiles = (N + 127) / 128, nk = (K + 63) / 64;
  const int64_t slots = static_cast<int64_t>(sms) * (nt <= 128 ? 2 : 1);
  if (nt == 0 || tiles >= slots) return 1;
  int64_t s = (slots * 7 / 8) / tiles;
  s = std::min<int64_t>(s, std::max<int64_t>(1, nk / 8));
  s = std::min<int64_t>(s, stream_max_splits(nt));
  return static_cast<int>(std::max<int64_t>(1, s));
}

// The split-K partials stay in the cluster's shared memory: no global scratch.
void stream_workspace(int64_t M, int64_t N, int64_t K, int sms, int64_t* ws_floats, int64_t* counters) {
  (void)M, (void)N, (void)K, (void)sms;
  *ws_floats = 0;
  *counters = 0;
}

// AXR_DENSE_TRACE=1: the stream kernel records 8 %globaltimer stamps per CTA into one
// device buffer (a measurement aid: entry, set-up done, first / last stage landed,
// accumulator ready, partials parked, epilogue done, exit); dense_trace() reads it back.
namespace {
unsigned long long* g_trace = nullptr;
int g_trace_ctas = 0;
bool trace_enabled() {
  static const bool on = [] {
    const char* e = getenv("AXR_DENSE_TRACE");
    return e && e[0] == '1';
  }();
  return on;
}
}  // namespace

int dense_trace(std::vector<unsigned long long>* out) {
  out->clear();
  if (!g_trace || g_trace_ctas == 0) return 0;
  out->resize(8ull * g_trace_ctas);
  if (cudaMemcpy(out->data(), g_trace, out->size() * 8, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  return g_trace_ctas;
}

std::string dense_gemm_launch(const DenseCall& c, cudaStream_t st) {
  if (c.M == 0 || c.N == 0) return "";
  if (c.K <= 0 || c.K % 8 != 0) return "K must be a positive multiple of 8";
  if ((reinterpret_cast<uintptr_t>(c.x) | reinterpret_cast<uintptr_t>(c.w)) % 16 != 0 || (c.ldx * 2) % 16 != 0 ||
      (c.ldw * 2) % 16 != 0)
    return "x / w must be 16-byte aligned with row strides of a multiple of 16 bytes";
  Args g{};
  g.M = c.M;
  g.N = c.N;
  g.K = c.K;
  g.err = c.err;
  g.e.out = reinterpret_cast<__nv_bfloat16*>(c.out);
  g.e.ldo = c.ldo;
  if (c.epi == kSwiGLU && c.N % 128 != 0) return "SwiGLU: N must be a multiple of 128";
  if (c.epi == kRope) {
    if (c.N != (c.Hq + 2 * c.Hkv) * 128) return "RoPE: N must be (Hq + 2 Hkv) * 128";
    if (!c.pos || !c.slots || !c.cos_sin || !c.kc || !c.vc || c.n_pos <= 0) return "RoPE: missing inputs";
    g.e.pos = c.pos;
    g.e.slots = c.slots;
    g.e.cos_sin = c.cos_sin;
    g.e.n_pos = c.n_pos;
    g.e.kc = reinterpret_cast<char*>(c.kc);
    g.e.vc = reinterpret_cast<char*>(c.vc);
    g.e.blk_stride = c.blk_stride;
    g.e.head_stride = c.head_stride;
    g.e.Hq = c.Hq;
    g.e.Hkv = c.Hkv;
  }
  if (c.epi == kResid) {
    if (!c.res) return "RESID: missing residual";
    g.e.res = reinterpret_cast<const __nv_bfloat16*>(c.res);
    g.e.ldr = c.ldr;
  }
  if (c.epi < kStore || c.epi > kRope) return "unknown epilogue";
  const int nt = stream_nt(c.M);
  cudaError_t e;
  if (nt != 0 && !c.force_big) {
    const int nk = (c.K + 63) / 64;
    g.splits = c.splits > 0 ? c.splits : stream_splits(c.M, c.N, c.K, sm_count(c.device));
    g.splits = std::max(1, std::min(std::min(g.splits, nk), stream_max_splits(nt)));
    CUtensorMap tw, tx;
    if (!make_map(&tw, c.w, c.N, c.K, c.ldw, 128) || !make_map(&tx, c.x, c.M, c.K, c.ldx, nt))
      return "cuTensorMapEncodeTiled failed";
    if (trace_enabled()) {
      const int ctas = ((c.N + 127) / 128) * g.splits;
      if (!g_trace) cudaMalloc(&g_trace, 8ull * 8 * 4096);
      g_trace_ctas = std::min(ctas, 4096);
      g.trace = ctas <= 4096 ? g_trace : nullptr;
    }
    switch (c.epi) {
      case kStore: e = launch_stream_nt<kStore>(nt, tw, tx, g, st); break;
      case kResid: e = launch_stream_nt<kResid>(nt, tw, tx, g, st); break;
      case kSwiGLU: e = launch_stream_nt<kSwiGLU>(nt, tw, tx, g, st); break;
      default: e = launch_stream_nt<kRope>(nt, tw, tx, g, st); break;
    }
  } else if (pair_enabled() && !c.force_one_cta) {
    CUtensorMap tx, tw;  // 128-row boxes: each CTA of a pair loads its half of the 256-row tile
    if (!make_map(&tx, c.x, c.M, c.K, c.ldx, 128) || !make_map(&tw, c.w, c.N, c.K, c.ldw, 128))
      return "cuTensorMapEncodeTiled failed";
    switch (c.epi) {
      case kStore: e = launch_pair<kStore>(tx, tw, g, c.device, st); break;
      case kResid: e = launch_pair<kResid>(tx, tw, g, c.device, st); break;
      case kSwiGLU: e = launch_pair<kSwiGLU>(tx, tw, g, c.device, st); break;
      default: e = launch_pair<kRope>(tx, tw, g, c.device, st); break;
    }
  } else {
    CUtensorMap tx, tw;
    if (!make_map(&tx, c.x, c.M, c.K, c.ldx, BM) || !make_map(&tw, c.w, c.N, c.K, c.ldw, BN))
      return "cuTensorMapEncodeTiled failed";
    switch (c.epi) {
      case kStore: e = launch_big<kStore>(tx, tw, g, c.device, st); break;
      case kResid: e = launch_big<kResid>(tx, tw, g, c.device, st); break;
      case kSwiGLU: e = launch_big<kSwiGLU>(tx, tw, g, c.device, st); break;
      default: e = launch_big<kRope>(tx, tw, g, c.device, st); break;
    }
  }
  if (e != cudaSuccess) return std::string("launch failed: ") + cudaGetErrorString(e);
  return "";
}

}  // namespace dense
}  // namespace axr
