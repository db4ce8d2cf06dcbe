// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), bf16
// paged KV cache, head_dim 128, GQA. One CTA = 256 query rows, as two 128-row sub-tiles
// A and B that ping-pong on the tensor core. A row is one (token, query head): either
// the rows of one head (gpack = 1), or -- for short suffixes over long prefixes -- the
// G = Hq / Hkv heads that share a KV head packed token-major (gpack = G), so a 128-token
// suffix fills both sub-tiles and every KV tile loaded serves G heads.
//
//   warp 8     TMA producer: K_j and V_j (128 tokens each) are gathered through the
//              block table as 8 pages x 2 halves of [16 tokens x 64 dims] boxes into a
//              ring of five 128-byte-swizzled [128 x 128] slots (K_0 V_0 K_1 V_1 ...).
//   warp 9     MMA issuer (one thread), per KV tile j:
//                PV_A(j), S_A(j+1), PV_B(j), S_B(j+1)
//              S_x = Q_x K^T goes to sub-tile x's TMEM S columns, O_x += P_x V (P_x read
//              from TMEM, V MN-major from shared memory) to its TMEM O columns.
//   warps 0-3 / 4-7   softmax of sub-tile A / B, one thread per query row (= TMEM
//              lane): S from TMEM, causal mask, running max, exp2, row sum, P (bf16
//              pairs) back into the first half of S's TMEM columns, where the PV MMA
//              reads it (P never touches shared memory, which leaves room for a
//              five-slot ring; with P in shared memory the ring had three slots and
//              K_{j+1} could only load once PV(j-1) was done, so the tensor pipe waited
//              on the load every tile). The running max only moves when a tile's
//              max exceeds it by more than 2^8 (O is then rescaled in TMEM), so the
//              exponentials stay below 256 and the rescale is rare.
//   epilogue   O / l from TMEM straight to the output rows.
//
// Ordering comes from tcgen05.commit, which fires only when every earlier MMA of the
// issuing thread has completed: when S_x(j+1) is ready, PV_x(j) is done, so the softmax
// may overwrite P_x and rescale O_x without further waits. S_x(j+1), which overwrites the
// TMEM columns holding P_x(j), is issued after PV_x(j) by the same thread, and one
// thread's MMAs execute in issue order. While one sub-tile's
// softmax runs, the tensor core works on the other's MMAs. Every mbarrier wait is
// bounded; on timeout the kernel records an error code, drains its own TMA loads and
// MMAs, frees TMEM and returns.
//
// Reference counterpart: the prefill attention the reference delegates to llama.cpp /
// vLLM library kernels; the reference has no prefill attention kernel of its own.
#include <cfloat>
#include <cstdlib>
#include <string>

#include "attn_combine.cuh"
#include "common.cuh"
#include "prefill_tc.h"
#include "tc_common.cuh"

namespace axr {
namespace fa {

constexpr int BM = 128, BN = 128, HD = 128;
constexpr int CHUNK = 128 * 128;  // one [128 rows x 64 bf16] swizzled chunk (16 KB)
constexpr int TILE = 2 * CHUNK;   // [128 x 128] bf16 tile (32 KB)
constexpr int RING = 5;           // K/V slots
constexpr int SMEM = 1024 + 2 * TILE /*Q_A,Q_B*/ + RING * TILE + 256;
constexpr int THREADS = 320;
constexpr float RESCALE_T = 8.f;  // log2 units

struct Params {
  const __nv_bfloat16* q;  // [T, Hq, 128]
  __nv_bfloat16* out;      // [T, Hq, 128]
  int Hq, Hkv;
  const int* block_table;
  int bt_stride;
  const int* cu_q;
  const int* seq_lens;
  float scale_log2;
  volatile int* err;
  int num_splits;   // KV slices per (query tile, head, sequence); 1 = no split
  int gpack;        // 1: grid.y = query heads; G = Hq/Hkv: grid.y = KV heads, rows = (token, head of the group)
  float* part_o;    // [T*Hq, S, 128] normalised partial outputs (S > 1 or partial_only)
  float* part_lse;  // [T*Hq, S] log2-domain log-sum-exps (S > 1 or partial_only)
  // Shared-prefix decode: every row sees all seq_lens[b] keys (no causal mask), row i's q
  // is row q_index[i] of q, and the result stays as partials for a later merge.
  int noncausal;
  const int* q_index;  // nullable: token i reads q row i
  int partial_only;
  long long* trace;    // AXR_PREFILL_TRACE=1: clock64 stamps of the CTA (0, 0, 0), 12 per KV tile
};

// byte offset of 16-byte unit u (0..15) of row r in a [128 x 128] bf16 K-major SW128 tile
__device__ __forceinline__ uint32_t swz_off(int r, int u) {
  return (u >> 3) * CHUNK + r * 128 + (((u & 7) ^ (r & 7)) << 4);
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic: one instruction for two values) and the
// three-input maximum: they halve the FMA-pipe instructions of the softmax.
__device__ __forceinline__ unsigned long long f2(float a, float b) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_split(unsigned long long x, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b, unsigned long long c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ unsigned long long f2_add(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ bool warp_ok(bool ok, volatile int* err) {
  return __all_sync(0xffffffffu, ok) && __shfl_sync(0xffffffffu, *err, 0) == 0;
}

__global__ void __launch_bounds__(THREADS, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap tmK,
                                                                const __grid_constant__ CUtensorMap tmV, Params p) {
  extern __shared__ __align__(1024) char fa_raw[];
  char* base = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(fa_raw) + 1023) & ~uintptr_t(1023));
  char* sQ = base;             // [2][TILE]
  char* sR = sQ + 2 * TILE;    // [RING][TILE]
  uint64_t* slot_full = reinterpret_cast<uint64_t*>(sR + RING * TILE);
  uint64_t* slot_free = slot_full + RING;
  uint64_t* s_full = slot_free + RING;  // [2] (A, B)
  uint64_t* p_full = s_full + 2;        // [2]
  uint64_t* o_done = p_full + 2;
  uint64_t* q_full = o_done + 1;
  uint64_t* drain = q_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // blocks start in x-fastest order: every head of the longest query tile (most KV tiles)
  // first, then the next tile, so the last CTAs to start are the short ones (measured
  // 0.84 against 0.98 ms for 8192 tokens x 32 heads with the tiles of one head first)
  const int tile_m = gridDim.y - 1 - blockIdx.y;
  const int S = p.num_splits;
  const int G = p.gpack;
  const int hy = blockIdx.x, b = blockIdx.z / S, split = blockIdx.z % S;
  const int q0 = p.cu_q[b], nq = p.cu_q[b + 1] - q0;
  const int nrow = nq * G;           // rows of this sequence: tokens x packed heads
  const int row0 = tile_m * 2 * BM;  // first row of sub-tile A
  if (row0 >= nrow) return;
  const bool has_b = row0 + BM < nrow;
  const int kv_len = p.seq_lens[b];
  const int pos0 = p.noncausal ? kv_len : kv_len - nq;  // absolute position of token 0
  const int kvh = G > 1 ? hy : hy / (p.Hq / p.Hkv);
  const int m_last = (min(nrow, row0 + 2 * BM) - 1) / G;  // last token of the tile
  const int kv_end = min(kv_len, pos0 + m_last + 1);
  const int n_all = (kv_end + BN - 1) / BN;
  // split-KV: this CTA takes KV tiles [t_begin, t_begin + n_tiles) of the query tile's range
  const int per = (n_all + S - 1) / S;
  const int t_begin = split * per;
  const int n_tiles = max(0, min(n_all, t_begin + per) - t_begin);
  if (n_tiles == 0) {  // no keys for this slice: mark its partials empty
    for (int r = threadIdx.x; p.part_lse != nullptr && r < 2 * BM; r += blockDim.x) {
      const int rr = row0 + r;
      if (rr < nrow) {
        const int head = G > 1 ? kvh * G + rr % G : hy;
        p.part_lse[((long long)(q0 + rr / G) * p.Hq + head) * S + split] = -FLT_MAX;
      }
    }
    return;
  }
  const int* bt = p.block_table + (long long)b * p.bt_stride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < RING; ++s) {
      tc::mbar_init(&slot_full[s], 1);
      tc::mbar_init(&slot_free[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&s_full[i], 1);
      tc::mbar_init(&p_full[i], 4);
    }
    tc::mbar_init(o_done, 1);
    tc::mbar_init(q_full, 8);
    tc::mbar_init(drain, 1);
    tc::fence_barrier_init();
    tc::prefetch_tmap(&tmK);
    tc::prefetch_tmap(&tmV);
  }
  if (warp == 9) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // TMEM columns: S_A 0-127, S_B 128-255, O_A 256-383, O_B 384-511

  if (warp == 8) {
    if (lane == 0) {  // ---------------- TMA producer: items K_0, V_0, K_1, V_1, ...
      int issued = 0;
      bool ok = true;
      long long* ptr = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) ? p.trace : nullptr;
      // The 8 block-table entries of a KV tile are read one tile ahead, as independent
      // loads: read next to the TMA issues (whose asm orders every memory access) they
      // were 8 dependent round trips per item and the ring ran dry (measured: a K tile
      // landed ~2600 cycles after issue, the MMA thread waited ~1200 of them every tile).
      int cur[8], nxt[8];
      auto page_ids = [&](int j, int (&o)[8]) {
#pragma unroll
        for (int pg = 0; pg < 8; ++pg) {
          const int tok = (t_begin + j) * BN + pg * 16;
          o[pg] = (j < n_tiles && tok < kv_len) ? bt[tok >> 4] : 0;
        }
      };
      page_ids(0, nxt);
      for (int i = 0; i < 2 * n_tiles; ++i) {
        const int s = i % RING, j = i >> 1;
        if ((i & 1) == 0) {  // K_j: its pages (shared with V_j) were read a tile ago
#pragma unroll
          for (int pg = 0; pg < 8; ++pg) cur[pg] = nxt[pg];
          page_ids(j + 1, nxt);
        }
        if (ptr && j < 128) ptr[j * 12 + 10 + (i & 1)] = clock64();
        if (i >= RING && !tc::mbar_wait(&slot_free[s], ((i / RING) + 1) & 1, p.err, 11)) { ok = false; break; }
        if (ptr && j < 128) ptr[j * 12 + 8 + (i & 1)] = clock64();
        const CUtensorMap* map = (i & 1) ? &tmV : &tmK;
        tc::mbar_arrive_expect_tx(&slot_full[s], TILE);
#pragma unroll
        for (int pg = 0; pg < 8; ++pg) {
          const int y = (cur[pg] * p.Hkv + kvh) * 16;
          tc::tma_load_2d(sR + s * TILE + pg * 2048, map, 0, y, &slot_full[s]);
          tc::tma_load_2d(sR + s * TILE + CHUNK + pg * 2048, map, 64, y, &slot_full[s]);
        }
        issued = i + 1;
      }
      if (!ok) {  // let this thread's loads land before the CTA can exit
        for (int i = max(0, issued - RING); i < issued; ++i) tc::mbar_wait_quiet(&slot_full[i % RING], (i / RING) & 1);
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {  // ---------------- MMA issuer
      constexpr uint32_t idesc_s = tc::idesc_bf16_f32(BM, BN);
      constexpr uint32_t idesc_pv = tc::idesc_bf16_f32_bmn(BM, HD);
      const int nsub = has_b ? 2 : 1;
      auto issue_s = [&](int x, int j) {  // S_x(j) = Q_x K_j^T
        const uint32_t q_addr = tc::smem_u32(sQ + x * TILE);
        const uint32_t k_addr = tc::smem_u32(sR + ((2 * j) % RING) * TILE);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK + (kk & 3) * 32;
          tc::mma_f16_ss(tmem + x * 128, tc::smem_desc_k_sw128(q_addr + off), tc::smem_desc_k_sw128(k_addr + off),
                         idesc_s, kk != 0);
        }
        tc::mma_commit(&s_full[x]);
      };
      auto issue_pv = [&](int x, int j) {  // O_x += P_x V_j, P_x (bf16) in TMEM over S_x's first 64 columns
        const uint32_t v_addr = tc::smem_u32(sR + ((2 * j + 1) % RING) * TILE);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          tc::mma_f16_ts(tmem + 256 + x * 128, tmem + x * 128 + kk * 8, tc::smem_desc_mn_sw128(v_addr + kk * 2048, CHUNK),
                         idesc_pv, (j | kk) != 0);
        }
      };
      long long* mtr = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) ? p.trace : nullptr;
      bool ok = tc::mbar_wait(q_full, 0, p.err, 12) && tc::mbar_wait(&slot_full[0], 0, p.err, 13);
      if (ok) {
        tc::tc_fence_after();
        for (int x = 0; x < nsub; ++x) issue_s(x, 0);
        tc::mma_commit(&slot_free[0]);  // K_0 consumed once the S MMAs complete
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int iv = 2 * j + 1, ik = 2 * j + 2;  // ring items V_j, K_{j+1}
        if (!tc::mbar_wait(&slot_full[iv % RING], (iv / RING) & 1, p.err, 14)) break;
        if (mtr && j < 128) mtr[j * 12 + 3] = clock64();  // V_j landed
        for (int x = 0; x < nsub; ++x) {
          if (!tc::mbar_wait(&p_full[x], j & 1, p.err, 16)) { ok = false; break; }
          if (mtr && j < 128) mtr[j * 12 + 4 * x + 2] = clock64();
          tc::tc_fence_after();
          issue_pv(x, j);
          if (j + 1 < n_tiles) {
            if (x == 0 && !tc::mbar_wait(&slot_full[ik % RING], (ik / RING) & 1, p.err, 15)) { ok = false; break; }
            if (mtr && x == 0 && j < 128) mtr[j * 12 + 7] = clock64();  // K_{j+1} landed
            tc::tc_fence_after();
            issue_s(x, j + 1);
          }
        }
        if (!ok) break;
        tc::mma_commit(&slot_free[iv % RING]);                    // V_j
        if (j + 1 < n_tiles) tc::mma_commit(&slot_free[ik % RING]);  // K_{j+1}
      }
      tc::mma_commit(o_done);
      tc::mma_commit(drain);
      tc::mbar_wait_quiet(drain, 0);  // every MMA of this CTA has completed
    }
  } else {
    // ---------------- softmax warps: 0-3 sub-tile A, 4-7 sub-tile B; thread = row = TMEM lane
    const int x = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + x * 128 + lane_off, tO = tmem + 256 + x * 128 + lane_off;
    const int qr = row0 + x * BM + row;  // row of the sequence
    const bool row_valid = qr < nrow;
    const int qt = row_valid ? qr / G : 0;  // its token
    const int hq = G > 1 ? kvh * G + qr % G : hy;
    const bool active = x == 0 || has_b;
    {
      const int src_tok = p.q_index != nullptr ? p.q_index[q0 + qt] : q0 + qt;
      const char* src = reinterpret_cast<const char*>(p.q + ((long long)src_tok * p.Hq + hq) * HD);
#pragma unroll
      for (int u = 0; u < 16; ++u) cp_async16_zfill(sQ + x * TILE + swz_off(row, u), src + u * 16, row_valid);
      cp_async_commit();
      cp_async_wait<0>();
      tc::fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(q_full);
    }
    const int qpos = pos0 + qt;
    const int qpos_min = pos0 + (row0 + x * BM) / G;
    // scores stay raw: the softmax scale (log2 units, > 0) enters the row maximum once and
    // every exponential through one FMA, 2^(c s - m)
    const float csc = p.scale_log2;
    float m_used = -INFINITY, l = 0.f;
    bool ok = active;
    long long* tr = (p.trace != nullptr && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && row == 0)
                        ? p.trace : nullptr;
    for (int j = 0; ok && j < n_tiles; ++j) {
      ok = warp_ok(tc::mbar_wait(&s_full[x], j & 1, p.err, 18), p.err);
      if (!ok) break;
      if (tr && j < 128) tr[j * 12 + 4 * x] = clock64();
      tc::tc_fence_after();
      float v[BN];
      {
        uint32_t r[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tc::tmem_ld32(tS + c * 32, r[c]);
        tc::tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) v[c * 32 + i] = __uint_as_float(r[c][i]);  // raw q.k

      }
      const int n0 = (t_begin + j) * BN;
      if (n0 + BN - 1 > qpos_min || n0 + BN > kv_len) {
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (n0 + i > qpos || n0 + i >= kv_len) v[i] = -INFINITY;
      }
      // row maximum as 8 independent chains of three-input maxima (a single 128-long
      // chain is latency-bound)
      float mx8[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) mx8[c] = max3(v[c], v[8 + c], v[16 + c]);
#pragma unroll
      for (int i = 24; i + 16 <= BN; i += 16)
#pragma unroll
        for (int c = 0; c < 8; ++c) mx8[c] = max3(mx8[c], v[i + c], v[i + 8 + c]);
#pragma unroll
      for (int c = 0; c < 8; ++c) mx8[c] = fmaxf(mx8[c], v[BN - 8 + c]);
      const float mt = csc * max3(max3(mx8[0], mx8[1], mx8[2]), max3(mx8[3], mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7]));
      if (j == 0) {
        m_used = mt;
      } else {
        // PV_x(j-1) completed before S_x(j) was signalled: O_x may be rescaled now
        const bool rescale = mt > m_used + RESCALE_T;
        if (__any_sync(0xffffffffu, rescale)) {
          const float alpha = rescale ? exp2f(m_used - mt) : 1.f;
          if (rescale) {
            m_used = mt;
            l *= alpha;
          }
#pragma unroll 1
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t r[32];
            tc::tmem_ld32(tO + c * 32, r);
            tc::tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
            tc::tmem_st32(tO + c * 32, r);
          }
          tc::tmem_st_wait();
        }
      }
      // masked scores are -inf: 2^(c (-inf) - m) is 0 for any finite m, and while every
      // score so far was masked (m = -inf) subtracting 0 gives 0 as well
      const float msub = m_used == -INFINITY ? 0.f : m_used;
      // exponent arguments c s - m and the row sum on packed pairs
      const unsigned long long sc2 = f2(csc, csc), ms2 = f2(-msub, -msub);
      unsigned long long l2[4] = {0ull, 0ull, 0ull, 0ull};  // +0.0f pairs
      // P as bf16 pairs into S_x's first 64 TMEM columns (S_x is already in registers), 16
      // columns per store; the PV MMA reads it from there as its A operand
#pragma unroll
      for (int u4 = 0; u4 < 4; ++u4) {
        uint32_t pk[16];
#pragma unroll
        for (int uu = 0; uu < 4; ++uu) {
          const int u = u4 * 4 + uu;
          float e[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float a, b;
            f2_split(f2_fma(f2(v[u * 8 + 2 * q], v[u * 8 + 2 * q + 1]), sc2, ms2), a, b);
            e[2 * q] = exp2f(a);
            e[2 * q + 1] = exp2f(b);
            l2[q] = f2_add(l2[q], f2(e[2 * q], e[2 * q + 1]));
            pk[uu * 4 + q] = pack_bf16x2(e[2 * q], e[2 * q + 1]);
          }
        }
        tc::tmem_st16(tS + u4 * 16, pk);
      }
      {
        float a0, b0, a1, b1, a2, b2, a3, b3;
        f2_split(l2[0], a0, b0);
        f2_split(l2[1], a1, b1);
        f2_split(l2[2], a2, b2);
        f2_split(l2[3], a3, b3);
        l += ((a0 + b0) + (a1 + b1)) + ((a2 + b2) + (a3 + b3));
      }
      tc::tmem_st_wait();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&p_full[x]);
      if (tr && j < 128) tr[j * 12 + 4 * x + 1] = clock64();
    }
    // ---------------- epilogue: O / l -> out
    if (ok) ok = warp_ok(tc::mbar_wait(o_done, 0, p.err, 21), p.err);
    if (ok && (S > 1 || p.partial_only)) {  // normalised partial output + log-sum-exp of this KV slice
      tc::tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const long long pr = ((long long)(q0 + qt) * p.Hq + hq) * S + split;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(tO + c * 32, r);
        tc::tmem_ld_wait();
        if (row_valid) {
          float4* dst = reinterpret_cast<float4*>(p.part_o + pr * HD + c * 32);
#pragma unroll
          for (int w4 = 0; w4 < 8; ++w4)
            dst[w4] = make_float4(__uint_as_float(r[4 * w4]) * inv, __uint_as_float(r[4 * w4 + 1]) * inv,
                                  __uint_as_float(r[4 * w4 + 2]) * inv, __uint_as_float(r[4 * w4 + 3]) * inv);
        }
      }
      if (row_valid) p.part_lse[pr] = l > 0.f ? m_used + __log2f(l) : -FLT_MAX;
    } else if (ok) {
      tc::tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = p.out + ((long long)(q0 + qt) * p.Hq + hq) * HD;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld32(tO + c * 32, r);
        tc::tmem_ld_wait();
        if (row_valid) {
#pragma unroll
          for (int w8 = 0; w8 < 4; ++w8) {
            const uint32_t* w = &r[w8 * 8];
            *reinterpret_cast<uint4*>(dst + c * 32 + w8 * 8) =
                make_uint4(pack_bf16x2(__uint_as_float(w[0]) * inv, __uint_as_float(w[1]) * inv),
                           pack_bf16x2(__uint_as_float(w[2]) * inv, __uint_as_float(w[3]) * inv),
                           pack_bf16x2(__uint_as_float(w[4]) * inv, __uint_as_float(w[5]) * inv),
                           pack_bf16x2(__uint_as_float(w[6]) * inv, __uint_as_float(w[7]) * inv));
          }
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 9) tc::tmem_dealloc(tmem, 512);
}

bool make_page_map(CUtensorMap* map, const void* ptr, int64_t rows) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(HD), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(HD * 2)};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t estr[2] = {1, 1};
  return cuTensorMapEncodeTiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box,
                                estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {
long long* g_prefill_trace = nullptr;
}

// Measurement aid (AXR_PREFILL_TRACE=1): clock64 stamps of the last launch's CTA (0, 0, 0),
// 12 per KV tile j: [softmax A: S ready, P stored; MMA: P_A seen; V_j landed; softmax B: S
// ready, P stored; MMA: P_B seen; K_{j+1} landed; producer: K_j issued, V_j issued, K_j slot
// wait started, V_j slot wait started].
int prefill_trace(long long* host, int n) {
  if (!g_prefill_trace) return 0;
  n = n < 12 * 128 ? n : 12 * 128;
  return cudaMemcpy(host, g_prefill_trace, n * sizeof(long long), cudaMemcpyDeviceToHost) == cudaSuccess ? n : -1;
}

std::string prefill_launch(const PrefillCall& c, cudaStream_t st) {
  if (c.B == 0 || c.max_q == 0) return "";
  if (c.Hq % c.Hkv != 0) return "Hq must be a multiple of Hkv";
  CUtensorMap tk, tv;
  if (!make_page_map(&tk, c.k, c.num_blocks * c.Hkv * 16) || !make_page_map(&tv, c.v, c.num_blocks * c.Hkv * 16))
    return "page regions must be 16-byte aligned (cuTensorMapEncodeTiled failed)";
  Params p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(c.q);
  p.out = reinterpret_cast<__nv_bfloat16*>(c.out);
  p.Hq = c.Hq;
  p.Hkv = c.Hkv;
  p.block_table = c.block_table;
  p.bt_stride = c.bt_stride;
  p.cu_q = c.cu_q;
  p.seq_lens = c.seq_lens;
  p.scale_log2 = c.scale * 1.4426950408889634f;
  p.err = c.err;
  const int S = c.num_splits > 1 ? c.num_splits : 1;
  p.num_splits = S;
  p.gpack = c.gqa_pack > 1 ? c.Hq / c.Hkv : 1;
  p.part_o = c.part_o;
  p.part_lse = c.part_lse;
  p.noncausal = c.noncausal != 0;
  p.partial_only = c.partial_only != 0;
  p.q_index = c.q_index;
  p.trace = nullptr;
  {
    static const bool on = [] {
      const char* e = getenv("AXR_PREFILL_TRACE");
      return e && e[0] == '1';
    }();
    if (on) {
      if (!g_prefill_trace) cudaMalloc(&g_prefill_trace, 12 * 128 * sizeof(long long));
      p.trace = g_prefill_trace;
    }
  }
  if ((S > 1 || p.partial_only) && (p.part_o == nullptr || p.part_lse == nullptr)) return "split-KV scratch missing";
  if ((int64_t)c.B * S >= 65536) return "too many sequences x splits";
  static bool attr = false;
  if (!attr) {
    const cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e);
    attr = true;
  }
  const int64_t rows = (int64_t)c.max_q * p.gpack;
  const int64_t tiles = (rows + 2 * BM - 1) / (2 * BM);
  const unsigned heads = p.gpack > 1 ? static_cast<unsigned>(c.Hkv) : static_cast<unsigned>(c.Hq);
  if (tiles >= 65536) return "too many query tiles";
  const dim3 grid(heads, static_cast<unsigned>(tiles), c.B * S);
  prefill_tc_kernel<<<grid, THREADS, SMEM, st>>>(tk, tv, p);
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) return std::string("launch failed: ") + cudaGetErrorString(e);
  if (S > 1 && c.T > 0 && !p.partial_only) {
    decode_combine_kernel<128><<<c.T * c.Hq, 128, 0, st>>>(p.part_o, p.part_lse, p.out, S);
    e = cudaPeekAtLastError();
    if (e != cudaSuccess) return std::string("combine launch failed: ") + cudaGetErrorString(e);
  }
  return "";
}

}  // namespace fa
}  // namespace axr
