// Causal flash attention (forward) with grouped-query heads for sm_100a, on tcgen05.
//
// Input is the packed projection qkv [B*S, (nq + 2*nkv) * D] (bf16): head h of q at columns
// [h*D, (h+1)*D), kv head g of k at [(nq+g)*D, ...) and of v at [(nq+nkv+g)*D, ...).  Output
// o [B*S, nq*D] (bf16) and lse [B, nq, S] (fp32, natural-log log-sum-exp of the scaled
// scores, consumed by the backward).
//
// One CTA computes 128 query rows of one (batch, q-head):
//   warp 8     TMA producer: Q once, then K_j / V_j into a 2-stage ring
//   warp 9     MMA issuer:   S_j = Q K_j^T into TMEM S[j%2]; O += P_j V_j into TMEM O
//   warps 0-7  softmax: two warps per TMEM lane quadrant (32 query rows), each owning 64 of
//              the 128 key columns; they exchange the row max through shared memory, keep
//              P_j relative to a lazily updated max (O in TMEM is rescaled only when the max
//              grows by more than 2^8), write P_j to shared memory (bf16, 128-byte swizzled
//              K-major tile) and finally store O / l and the LSE.
// TMEM: S0, S1 (2 x 128 fp32 columns), O (D columns).  Causal masking only touches the
// diagonal block; blocks past the diagonal are skipped.  Every mbarrier wait is bounded.
//
// Reference: the reference calls torch SDPA (femtotron/model/llama_partial_model.py:70).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tmap.h"

#include <cstdlib>
#include <string>

namespace ft {
namespace fa {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int NTHREADS = 320;  // 8 softmax warps, 1 TMA warp, 1 MMA warp
constexpr int PRODUCER_WARP = 8, MMA_WARP = 9;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  int B, S, nq, nkv, D;
  __nv_bfloat16* O;
  int64_t ldo;
  float* lse;
  float scale_log2;  // softmax scale * log2(e)
  int nqb;           // query blocks per sequence
  int* err;
};

__device__ __forceinline__ uint64_t gns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool wait_b(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = gns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (gns() - t0 > 2000000000ull) {
      if (err) atomicExch(err, code);
      return false;
    }
  }
}

template <int D>
struct Smem {
  // every operand tile is stored as D/64 chunks of [128 rows][64 bf16] (128-byte swizzle)
  __nv_bfloat16 q[BQ * D];
  __nv_bfloat16 k[2][BKV * D];
  __nv_bfloat16 v[2][BKV * D];
  __nv_bfloat16 p[2][BQ * BKV];
  uint64_t q_full;
  uint64_t k_full[2], v_full[2], kv_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2];
  // o_ready[j & 1] completes when P V product j (and every earlier MMA) is done; a consumer
  // never lags a barrier by two phases, so parity waits on it are exact
  uint64_t o_ready[2];
  // row max of each column half, exchanged between the two warps of a row; reused for the
  // final partial sums (after the last block both halves are done reading it)
  float red_max[2][BQ];
  uint32_t tmem_base;
};

// Largest growth of a row's running max (log2 units) before the accumulated output is
// rescaled: probabilities stay below 2^8 relative to the stale max, which bf16 P and the
// fp32 accumulator absorb, so most blocks need no rescale pass over O.
constexpr float kRescaleThreshold = 8.0f;

template <int D>
__global__ void __launch_bounds__(NTHREADS, 1)
    flash_fwd_kernel(const __grid_constant__ CUtensorMap tm_qkv, const Params p) {
  using Sm = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  Sm& s = *reinterpret_cast<Sm*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // heaviest (latest) query blocks first for causal load balance
  // (every head's first wave holds the longest rows, so the short ones fill the tail)
  const int qb = p.nqb - 1 - static_cast<int>(blockIdx.y);
  const int bh = blockIdx.x;
  const int b = bh / p.nq, h = bh % p.nq;
  const int g = h / (p.nq / p.nkv);
  const int row0 = b * p.S + qb * BQ;          // first token row of this query block
  const int kv_row0 = b * p.S;
  const int nblocks = qb + 1;                  // causal: key blocks 0..qb
  const int qcol = h * D, kcol = (p.nq + g) * D, vcol = (p.nq + p.nkv + g) * D;
  constexpr int CH = D / 64;                   // 64-wide chunks along the head dim
  constexpr uint32_t TILE_BYTES = 128 * D * 2;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
      mbar_init(&s.s_full[i], 1);
      mbar_init(&s.s_free[i], 8);
      mbar_init(&s.p_full[i], 8);
      mbar_init(&s.o_ready[i], 1);
    }
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  auto tS = [tmem](int st) -> uint32_t { return tmem + (st ? 128u : 0u); };
  const uint32_t tO = tmem + 256;

  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      prefetch_tmap(&tm_qkv);
      mbar_arrive_expect_tx(&s.q_full, TILE_BYTES);
#pragma unroll
      for (int c = 0; c < CH; ++c) tma_load_2d(s.q + c * 128 * 64, &tm_qkv, &s.q_full, qcol + c * 64, row0);
      for (int j = 0; j < nblocks; ++j) {
        const int st = j & 1;
        if (!wait_b(&s.kv_empty[st], ((j >> 1) & 1) ^ 1, p.err, 21)) break;
        const int kr = kv_row0 + j * BKV;
        mbar_arrive_expect_tx(&s.k_full[st], TILE_BYTES);
#pragma unroll
        for (int c = 0; c < CH; ++c)
          tma_load_2d(s.k[st] + c * 128 * 64, &tm_qkv, &s.k_full[st], kcol + c * 64, kr);
        mbar_arrive_expect_tx(&s.v_full[st], TILE_BYTES);
#pragma unroll
        for (int c = 0; c < CH; ++c)
          tma_load_2d(s.v[st] + c * 128 * 64, &tm_qkv, &s.v_full[st], vcol + c * 64, kr);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc_bf16(128, BKV, false, false);  // Q (K-major) x K (K-major)
      constexpr uint32_t idO = make_idesc_bf16(128, D, false, true);     // P (K-major) x V (MN-major)
      bool ok = wait_b(&s.q_full, 0, p.err, 22);
      const uint32_t qa = smem_u32(s.q);
      auto issue_pv = [&](int j) -> bool {
        const int st = j & 1;
        if (!wait_b(&s.p_full[st], (j >> 1) & 1, p.err, 23)) return false;
        if (!wait_b(&s.v_full[st], (j >> 1) & 1, p.err, 24)) return false;
        tc_fence_after();
        const uint32_t va = smem_u32(s.v[st]);
        const uint32_t pa = smem_u32(s.p[st]);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          // A = P: K (keys) chunks of 64, 32 bytes per 16 keys inside a chunk
          const uint64_t ad = make_sw128_desc(pa + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
          // B = V: MN-major (head dim contiguous), 16 key rows = 2048 bytes per step
          const uint64_t bd = make_sw128_desc(va + kk * 2048, 128 * 128, 1024);
          mma_bf16(tO, ad, bd, idO, (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&s.kv_empty[st]);
        mma_commit(&s.o_ready[st]);
        return true;
      };
      for (int j = 0; j < nblocks && ok; ++j) {
        const int st = j & 1;
        if (!wait_b(&s.k_full[st], (j >> 1) & 1, p.err, 26)) { ok = false; break; }
        if (!wait_b(&s.s_free[st], ((j >> 1) & 1) ^ 1, p.err, 27)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ka = smem_u32(s.k[st]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 128 * 128 + (kk & 3) * 32;
          mma_bf16(tS(st), make_sw128_desc(qa + off, 16, 1024), make_sw128_desc(ka + off, 16, 1024),
                   idS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.s_full[st]);
        if (j >= 1 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) issue_pv(nblocks - 1);
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..7
    // Warps q and q+4 own the same 32 query rows (TMEM lane quadrant q) and split the 128
    // key columns (half = warp / 4); the two threads of a row exchange only the row max
    // each block (named barrier per warp pair) and their partial sums at the end.
    const int quad = warp & 3, half = warp >> 2;
    const int r = quad * 32 + lane;          // query row within the block (TMEM lane)
    const int qpos = qb * BQ + r;            // position within the sequence
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int col0 = half * (BKV / 2);       // this thread's 64 key columns
    float m_used = -INFINITY, l_run = 0.f;   // max the probabilities are relative to, own-half sum
    bool ok = true;
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + quad) : "memory"); };
    // wait until P V product `pv` has completed (barrier o_ready[pv & 1], phase pv >> 1)
    auto wait_pv = [&](int pv) -> bool {
      return pv < 0 || wait_b(&s.o_ready[pv & 1], (pv >> 1) & 1, p.err, 28);
    };

    // Both warps of a row pair execute every pair barrier even after a failed (timed-out)
    // wait, so a failure can never strand the partner on an unbounded named barrier.
    for (int j = 0; j < nblocks; ++j) {
      const int st = j & 1;
      if (ok && !wait_b(&s.s_full[st], (j >> 1) & 1, p.err, 29)) ok = false;
      // P buffer `st` is free once product j-2 (which read it) is done
      if (ok && !wait_pv(j - 2)) ok = false;
      tc_fence_after();
      const bool diag = (j == qb);
      uint32_t sv[BKV / 2];
      float mloc = -INFINITY;
      if (ok) {
        tmem_ld_32x32b_x32(tS(st) + lane_off + col0, *reinterpret_cast<uint32_t(*)[32]>(sv));
        tmem_ld_32x32b_x32(tS(st) + lane_off + col0 + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.s_free[st]);  // S buffer may be overwritten
        // row max of the raw scores (the scale is positive, so it commutes with max); on the
        // diagonal block, keys after the query are replaced by -inf
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        if (diag) {
          const int lim = qpos - (j * BKV + col0);  // keys i <= lim are visible
#pragma unroll
          for (int i = 0; i < BKV / 2; ++i) {
            if (i > lim) sv[i] = __float_as_uint(-INFINITY);
            mx4[i & 3] = fmaxf(mx4[i & 3], __uint_as_float(sv[i]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < BKV / 2; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], __uint_as_float(sv[i]));
        }
        mloc = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      }
      s.red_max[half][r] = mloc;
      pair_sync();
      const float mx = fmaxf(s.red_max[0][r], s.red_max[1][r]);
      pair_sync();  // both halves read before the next block overwrites
      if (!ok) continue;
      // lazy rescale of the TMEM accumulator (same decision in both halves of a row)
      const bool need = (m_used == -INFINITY) || (mx - m_used > kRescaleThreshold);
      const float m_new = need ? fmaxf(m_used, mx) : m_used;
      const float alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - m_new);
      if (j > 0 && __any_sync(0xffffffff, need)) {
        if (!wait_pv(j - 1)) { ok = false; continue; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {  // this half's D/2 output columns
          uint32_t ov[16];
          const uint32_t ta = tO + lane_off + half * (D / 2) + c * 16;
          tmem_ld_32x32b_x16(ta, ov);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
          tmem_st_32x32b_x16(ta, ov);
        }
        tmem_wait_st();
      }
      l_run *= alpha;
      m_used = m_new;
      // probabilities relative to m_used, bf16, into this half's chunk of the swizzled P tile
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      uint8_t* rowp = reinterpret_cast<uint8_t*>(s.p[st]) + half * 128 * 128 + r * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          // p = 2^(s * scale - m) as one FMA feeding exp2
          const float e0 = exp2f(fmaf(__uint_as_float(sv[c * 32 + i]), p.scale_log2, -m_used));
          const float e1 = exp2f(fmaf(__uint_as_float(sv[c * 32 + i + 1]), p.scale_log2, -m_used));
          sum4[(i >> 1) & 3] += e0 + e1;
          const __nv_bfloat162 bp = __floats2bfloat162_rn(e0, e1);
          pk[i >> 1] = *reinterpret_cast<const uint32_t*>(&bp);
        }
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int jj = (c * 4 + q4) ^ (r & 7);
          *reinterpret_cast<uint4*>(rowp + jj * 16) =
              make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
        }
      }
      l_run += (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full[st]);
    }
    if (ok) ok = wait_pv(nblocks - 1);
    // epilogue: O / l to bf16 (each half writes D/2 columns), LSE (natural log)
    s.red_max[half][r] = l_run;
    pair_sync();
    if (ok) {
      tc_fence_after();
      const float l = s.red_max[0][r] + s.red_max[1][r];
      const float inv = 1.f / l;
      __nv_bfloat16* orow = p.O + static_cast<int64_t>(row0 + r) * p.ldo + h * D + half * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[16];
        tmem_ld_32x32b_x16(tO + lane_off + half * (D / 2) + c * 16, ov);
        tmem_wait_ld();
        uint4 q0, q1;
        q0.x = pack_bf16x2(__uint_as_float(ov[0]) * inv, __uint_as_float(ov[1]) * inv);
        q0.y = pack_bf16x2(__uint_as_float(ov[2]) * inv, __uint_as_float(ov[3]) * inv);
        q0.z = pack_bf16x2(__uint_as_float(ov[4]) * inv, __uint_as_float(ov[5]) * inv);
        q0.w = pack_bf16x2(__uint_as_float(ov[6]) * inv, __uint_as_float(ov[7]) * inv);
        q1.x = pack_bf16x2(__uint_as_float(ov[8]) * inv, __uint_as_float(ov[9]) * inv);
        q1.y = pack_bf16x2(__uint_as_float(ov[10]) * inv, __uint_as_float(ov[11]) * inv);
        q1.z = pack_bf16x2(__uint_as_float(ov[12]) * inv, __uint_as_float(ov[13]) * inv);
        q1.w = pack_bf16x2(__uint_as_float(ov[14]) * inv, __uint_as_float(ov[15]) * inv);
        *reinterpret_cast<uint4*>(orow + 16 * c) = q0;
        *reinterpret_cast<uint4*>(orow + 16 * c + 8) = q1;
      }
      if (half == 0)
        p.lse[(static_cast<int64_t>(b) * p.nq + h) * p.S + qpos] = (m_used + log2f(l)) / kLog2e;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fa

// ------------------------------------------------------------------------------------------
// Two query tiles per CTA ("ping-pong").  One CTA computes query blocks 2c and 2c+1 of one
// (batch, q-head); they share every K_j / V_j tile.  Warps 0-3 run the softmax of tile 0,
// warps 4-7 that of tile 1, each thread owning one full query row (no cross-warp max
// exchange).  The MMA warp interleaves the tiles
//     S0(0) S1(0) | PV0(0) S0(1) PV1(0) S1(1) | PV0(1) S0(2) PV1(1) S1(2) | ...
// so the tensor core works on one tile while the other tile's softmax runs.  TMEM holds
// S0, S1, O0, O1 (4 x 128 fp32 columns).  P_t is written as packed bf16 pairs over the first
// 64 columns of S_t (already read) and the P V product takes its A operand from TMEM, so
// shared memory carries only Q, K and V: the Q K^T product reads 64 KB per 128x128 block and
// P V only V's 32 KB (with P in shared memory both products sat at the 128 B/clk shared-
// memory read limit).  S_t(j+1) is issued after P_t(j) V_j by the same thread, and
// tcgen05.mma operations from one thread execute in issue order, so the product that
// overwrites S_t never overtakes the one reading P_t.  The P V product of a tile starts on
// keys 0..63 while the softmax still computes keys 64..127.  K and V share a 4-stage TMA ring.
// A quarter of the exponentials (key columns 3 mod 4) run on the FMA pipe (exp2_poly) so the
// special-function unit, which otherwise sets the pace of the softmax, has slack.
namespace fa2 {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int NTHREADS = 320;  // 8 softmax warps, 1 TMA warp, 1 MMA warp
constexpr int PRODUCER_WARP = 8, MMA_WARP = 9;
constexpr int KV_STAGES = 4;

template <int D>
struct Smem {
  __nv_bfloat16 q[2][BQ * D];
  __nv_bfloat16 kv[KV_STAGES][BKV * D];  // ring of K_0, V_0, K_1, V_1, ...
  uint64_t q_full;
  uint64_t kv_full[KV_STAGES], kv_empty[KV_STAGES];
  uint64_t s_full[2], s_free[2], p_full[2], o_done[2];
  uint64_t p_half[2];   // keys 0..63 of P_t(j) stored: the P V product may start on them
  uint32_t tmem_base;
};

// 2^x on the FMA pipe, for x <= 2^8.  Cody-Waite reduction x = n + f with n = rint(x) taken
// from the fp32 sum x + 1.5*2^23 (round-to-nearest puts n in the low mantissa bits) and
// f in [-1/2, 1/2]; 2^f from a degree-3 polynomial fitted here to minimise the maximum
// relative error on [-1/2, 1/2] (linear-programming minimax over 4001 points: 7.5e-5, far
// below bf16's 2^-9); n is added to the exponent field.  x is clamped at -125 so the
// exponent field stays normal (masked keys are zeroed by the caller).
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.f);
  constexpr float kShift = 12582912.f;  // 1.5 * 2^23
  const float t = x + kShift;
  const float n = t - kShift;
  const float f = x - n;
  float q = fmaf(fmaf(fmaf(0.0551716685f, f, 0.2426111251f), f, 0.6932609677f), f, 0.9999280572f);
  const int ni = __float_as_int(t) - __float_as_int(kShift);
  return __int_as_float(__float_as_int(q) + (ni << 23));
}

__device__ __forceinline__ float ex2_sfu(float x) { return ex2_approx(x); }

// Three-input fp32 max (sm_100 max.f32 with three sources).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Probabilities of 32 keys (columns c0..c0+31 of this thread's row, scores sv[c0..c0+31]):
// p = 2^(s*scale - m), packed bf16 pairs into pk, row sums into sum4.  MASK (diagonal block
// only) zeroes keys after the query row r; EMU sends keys 3 mod 4 to exp2_poly.
template <bool MASK, bool EMU>
__device__ __forceinline__ void probs32(const uint32_t* sv, int c0, int r, float scale, float m,
                                        float (&sum4)[4], uint32_t (&pk)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float x0 = fmaf(__uint_as_float(sv[c0 + 2 * e]), scale, -m);
    const float x1 = fmaf(__uint_as_float(sv[c0 + 2 * e + 1]), scale, -m);
    float e0 = ex2_sfu(x0);
    float e1 = (EMU && (e & 1)) ? exp2_poly(x1) : ex2_sfu(x1);
    if (MASK) {
      e0 = (c0 + 2 * e > r) ? 0.f : e0;
      e1 = (c0 + 2 * e + 1 > r) ? 0.f : e1;
    }
    sum4[e & 3] += e0 + e1;
    pk[e] = pack_bf16x2(e0, e1);
  }
}

template <int D, bool EMU, bool ONE_PASS>
__global__ void __launch_bounds__(NTHREADS, 1)
    flash_fwd_pp_kernel(const __grid_constant__ CUtensorMap tm_qkv, const fa::Params p) {
  using Sm = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  Sm& s = *reinterpret_cast<Sm*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // heaviest query-block pairs first (causal load balance)
  const int nqb2 = p.nqb / 2;
  const int qb2 = nqb2 - 1 - static_cast<int>(blockIdx.y);
  const int bh = blockIdx.x;
  const int b = bh / p.nq, h = bh % p.nq;
  const int g = h / (p.nq / p.nkv);
  const int row0 = b * p.S + qb2 * 2 * BQ;     // first token row of tile 0
  const int kv_row0 = b * p.S;
  const int n1 = 2 * qb2 + 2;                  // key blocks seen by tile 1 (tile 0: n1 - 1)
  const int n0 = n1 - 1;
  const int qcol = h * D, kcol = (p.nq + g) * D, vcol = (p.nq + p.nkv + g) * D;
  constexpr int CH = D / 64;
  constexpr uint32_t TILE_BYTES = 128 * D * 2;

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s.s_full[t], 1);
      mbar_init(&s.s_free[t], 4);
      mbar_init(&s.p_full[t], 4);
      mbar_init(&s.p_half[t], 4);
      mbar_init(&s.o_done[t], 1);
    }
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  auto tS = [tmem](int t) -> uint32_t { return tmem + static_cast<uint32_t>(t) * 128u; };
  auto tO = [tmem](int t) -> uint32_t { return tmem + 256u + static_cast<uint32_t>(t) * 128u; };

  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      prefetch_tmap(&tm_qkv);
      mbar_arrive_expect_tx(&s.q_full, 2 * TILE_BYTES);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < CH; ++c)
          tma_load_2d(s.q[t] + c * 128 * 64, &tm_qkv, &s.q_full, qcol + c * 64, row0 + t * BQ);
      for (int item = 0; item < 2 * n1; ++item) {
        const int st = item % KV_STAGES, j = item >> 1;
        if (!fa::wait_b(&s.kv_empty[st], ((item / KV_STAGES) & 1) ^ 1, p.err, 41)) break;
        const int col = (item & 1) ? vcol : kcol;
        mbar_arrive_expect_tx(&s.kv_full[st], TILE_BYTES);
#pragma unroll
        for (int c = 0; c < CH; ++c)
          tma_load_2d(s.kv[st] + c * 128 * 64, &tm_qkv, &s.kv_full[st], col + c * 64, kv_row0 + j * BKV);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc_bf16(128, BKV, false, false);  // Q (K-major) x K (K-major)
      constexpr uint32_t idO = make_idesc_bf16(128, D, false, true);     // P (K-major) x V (MN-major)
      auto kv_wait = [&](int item) -> bool {
        return fa::wait_b(&s.kv_full[item % KV_STAGES], (item / KV_STAGES) & 1, p.err, 42);
      };
      // S_t(j) = Q_t K_j^T once the softmax has read S_t(j-1)
      auto issue_s = [&](int t, int j) -> bool {
        if (!fa::wait_b(&s.s_free[t], (j & 1) ^ 1, p.err, 43)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(s.q[t]), ka = smem_u32(s.kv[(2 * j) % KV_STAGES]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 128 * 128 + (kk & 3) * 32;
          mma_bf16(tS(t), make_sw128_desc(qa + off, 16, 1024), make_sw128_desc(ka + off, 16, 1024),
                   idS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.s_full[t]);
        return true;
      };
      // O_t += P_t(j) V_j once the softmax has written P_t(j) (A = P from TMEM: 16 keys =
      // 8 packed columns per MMA; B = V, MN-major: 16 key rows = 2048 bytes per MMA)
      // The first half (keys 0..63) starts as soon as the softmax has stored it.
      auto issue_pv = [&](int t, int j) -> bool {
        const uint32_t va = smem_u32(s.kv[(2 * j + 1) % KV_STAGES]);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if (!fa::wait_b(half ? &s.p_full[t] : &s.p_half[t], j & 1, p.err, 44)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = half * 4; kk < half * 4 + 4; ++kk) {
            const uint64_t bd = make_sw128_desc(va + kk * 2048, 128 * 128, 1024);
            mma_bf16_ts(tO(t), tS(t) + kk * 8, bd, idO, (j > 0 || kk > 0) ? 1u : 0u);
          }
        }
        mma_commit(&s.o_done[t]);
        return true;
      };
      bool ok = fa::wait_b(&s.q_full, 0, p.err, 45) && kv_wait(0) && issue_s(0, 0) && issue_s(1, 0);
      if (ok) mma_commit(&s.kv_empty[0]);  // K_0 is free once S0(0) and S1(0) complete
      for (int j = 0; ok && j < n1; ++j) {
        const int iv = 2 * j + 1, ik = 2 * j + 2;  // ring items of V_j and K_{j+1}
        if (j < n0) {
          ok = kv_wait(iv) && issue_pv(0, j);
          if (ok && j + 1 < n0) ok = kv_wait(ik) && issue_s(0, j + 1);
          if (!ok) break;
        }
        ok = kv_wait(iv) && issue_pv(1, j);
        if (!ok) break;
        mma_commit(&s.kv_empty[iv % KV_STAGES]);
        if (j + 1 < n1) {
          ok = kv_wait(ik) && issue_s(1, j + 1);
          if (!ok) break;
          mma_commit(&s.kv_empty[ik % KV_STAGES]);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ softmax warps 0..7
    const int t = warp >> 2, quad = warp & 3;
    const int r = quad * 32 + lane;            // query row within the tile (TMEM lane)
    const int qblk = 2 * qb2 + t;
    const int qpos = qblk * BQ + r;            // position within the sequence
    const int nt = qblk + 1;                   // key blocks 0..qblk
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    float m_used = -INFINITY, l_run = 0.f;
    bool ok = true;
    // ONE_PASS: each thread reads its row of S_t once (128 fp32 columns into registers), takes
    // the row max, then writes the probabilities 32 keys at a time as packed bf16 pairs over
    // the first 64 columns of S_t (every score is already in registers, so nothing is read
    // after it is overwritten).  Otherwise the row is read twice (all of it for the max, then
    // 64 columns at a time for the probabilities), which needs fewer registers.  S_t cannot
    // be overwritten before P_t is written anyway (the MMA warp issues S_t(j+1) after
    // P_t(j) V_j), so the second read costs no overlap.  Only the diagonal block (one in
    // S/128 per row) runs the masked code.
    for (int j = 0; j < nt && ok; ++j) {
      ok = __all_sync(0xffffffffu, fa::wait_b(&s.s_full[t], j & 1, p.err, 46));
      if (!ok) break;
      tc_fence_after();
      const bool diag = (j == qblk);   // keys after the query (column > r) are masked
      uint32_t sv[ONE_PASS ? BKV : 1];
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      {
        uint32_t sa[ONE_PASS ? 1 : BKV];
        uint32_t* sr = ONE_PASS ? sv : sa;
#pragma unroll
        for (int c = 0; c < BKV; c += 32)
          tmem_ld_32x32b_x32(tS(t) + lane_off + c, *reinterpret_cast<uint32_t(*)[32]>(sr + c));
        tmem_wait_ld();
        if (diag) {
#pragma unroll
          for (int i = 0; i < BKV; i += 2)
            mx4[(i >> 1) & 3] = max3f(mx4[(i >> 1) & 3], i > r ? -INFINITY : __uint_as_float(sr[i]),
                                      i + 1 > r ? -INFINITY : __uint_as_float(sr[i + 1]));
        } else {
#pragma unroll
          for (int i = 0; i < BKV; i += 2)
            mx4[(i >> 1) & 3] = max3f(mx4[(i >> 1) & 3], __uint_as_float(sr[i]), __uint_as_float(sr[i + 1]));
        }
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
      const bool need = (m_used == -INFINITY) || (mx - m_used > fa::kRescaleThreshold);
      const float m_new = need ? fmaxf(m_used, mx) : m_used;
      const float alpha = (m_used == -INFINITY) ? 0.f : exp2f(m_used - m_new);
      // O_t is stable and P_t is free once P V product j-1 of this tile has completed
      if (j > 0) {
        ok = __all_sync(0xffffffffu, fa::wait_b(&s.o_done[t], (j - 1) & 1, p.err, 47));
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int c = 0; c < D / 16; ++c) {
            uint32_t ov[16];
            const uint32_t ta = tO(t) + lane_off + c * 16;
            tmem_ld_32x32b_x16(ta, ov);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) ov[i] = __float_as_uint(__uint_as_float(ov[i]) * alpha);
            tmem_st_32x32b_x16(ta, ov);
          }
          tmem_wait_st();
        }
      }
      l_run *= alpha;
      m_used = m_new;
      // P = 2^(s * scale - m): keys 32q..32q+31 as packed pairs into columns 16q..16q+15
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      if constexpr (ONE_PASS) {
#pragma unroll
        for (int q = 0; q < BKV / 32; ++q) {
          uint32_t pk[16];
          if (diag) probs32<true, EMU>(sv, q * 32, r, p.scale_log2, m_used, sum4, pk);
          else probs32<false, EMU>(sv, q * 32, r, p.scale_log2, m_used, sum4, pk);
          tmem_st_32x32b_x16(tS(t) + lane_off + q * 16, pk);
          if (q == 1) {   // keys 0..63 stored
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.p_half[t]);
          }
        }
      } else {
#pragma unroll
        for (int cc = 0; cc < BKV / 64; ++cc) {
          uint32_t sb[64];
          tmem_ld_32x32b_x32(tS(t) + lane_off + cc * 64, *reinterpret_cast<uint32_t(*)[32]>(sb));
          tmem_ld_32x32b_x32(tS(t) + lane_off + cc * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(sb + 32));
          tmem_wait_ld();
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t pk[16];
            if (diag) probs32<true, EMU>(sb + h2 * 32, 0, r - cc * 64 - h2 * 32, p.scale_log2, m_used, sum4, pk);
            else probs32<false, EMU>(sb + h2 * 32, 0, 0, p.scale_log2, m_used, sum4, pk);
            tmem_st_32x32b_x16(tS(t) + lane_off + cc * 32 + h2 * 16, pk);
          }
          if (cc == 0) {   // keys 0..63 stored
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.p_half[t]);
          }
        }
      }
      tmem_wait_st();
      l_run += (sum4[0] + sum4[1]) + (sum4[2] + sum4[3]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.s_free[t]);   // S_t(j) fully read
        mbar_arrive(&s.p_full[t]);   // P_t(j) stored in TMEM
      }
    }
    if (ok) ok = __all_sync(0xffffffffu, fa::wait_b(&s.o_done[t], (nt - 1) & 1, p.err, 48));
    if (ok) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      __nv_bfloat16* orow = p.O + static_cast<int64_t>(row0 + t * BQ + r) * p.ldo + h * D;
#pragma unroll
      for (int c = 0; c < D / 16; ++c) {
        uint32_t ov[16];
        tmem_ld_32x32b_x16(tO(t) + lane_off + c * 16, ov);
        tmem_wait_ld();
        uint4 q0, q1;
        q0.x = pack_bf16x2(__uint_as_float(ov[0]) * inv, __uint_as_float(ov[1]) * inv);
        q0.y = pack_bf16x2(__uint_as_float(ov[2]) * inv, __uint_as_float(ov[3]) * inv);
        q0.z = pack_bf16x2(__uint_as_float(ov[4]) * inv, __uint_as_float(ov[5]) * inv);
        q0.w = pack_bf16x2(__uint_as_float(ov[6]) * inv, __uint_as_float(ov[7]) * inv);
        q1.x = pack_bf16x2(__uint_as_float(ov[8]) * inv, __uint_as_float(ov[9]) * inv);
        q1.y = pack_bf16x2(__uint_as_float(ov[10]) * inv, __uint_as_float(ov[11]) * inv);
        q1.z = pack_bf16x2(__uint_as_float(ov[12]) * inv, __uint_as_float(ov[13]) * inv);
        q1.w = pack_bf16x2(__uint_as_float(ov[14]) * inv, __uint_as_float(ov[15]) * inv);
        *reinterpret_cast<uint4*>(orow + 16 * c) = q0;
        *reinterpret_cast<uint4*>(orow + 16 * c + 8) = q1;
      }
      p.lse[(static_cast<int64_t>(b) * p.nq + h) * p.S + qpos] = (m_used + log2f(l_run)) / fa::kLog2e;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fa2

// variant: 0 = automatic (the two-tile kernel whenever S is a multiple of 256, unless the
// environment sets FT_FA_FWD=v1), 1 = one-tile kernel, 2 = two-tile kernel reading each row of
// S twice from TMEM (fewest registers; measured fastest), 3 = two-tile kernel reading the row
// once (168 registers, small spill), 4 = as 3 with a quarter of the exponentials on the FMA
// pipe.  Every exponential of variants 2 and 3 runs on the special-function unit.
void flash_fwd_variant(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B,
                       int64_t S, int64_t nq, int64_t nkv, int64_t D, torch::Tensor& err,
                       int64_t variant) {
  using namespace fa;
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1);
  TORCH_CHECK(D == 64 || D == 128, "flash_fwd: head_dim 64 or 128");
  TORCH_CHECK(S % 128 == 0, "flash_fwd: sequence length must be a multiple of 128");
  TORCH_CHECK(nq % nkv == 0, "flash_fwd: q heads must be a multiple of kv heads");
  TORCH_CHECK(qkv.size(0) == B * S && qkv.size(1) >= (nq + 2 * nkv) * D);
  TORCH_CHECK(o.stride(1) == 1 && o.stride(0) % 8 == 0 && lse.is_contiguous());
  const c10::cuda::CUDAGuard g(qkv.device());
  CUtensorMap tm = make_tmap_2d(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv.size(1),
                                qkv.size(0), qkv.stride(0), 64, 128, true);
  Params p;
  p.B = B; p.S = S; p.nq = nq; p.nkv = nkv; p.D = D;
  p.O = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  p.ldo = o.stride(0);
  p.lse = lse.data_ptr<float>();
  p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D))) * kLog2e;
  p.nqb = S / 128;
  p.err = err.data_ptr<int>();
  auto st = at::cuda::getCurrentCUDAStream();
  static const bool force_v1 = [] { const char* e = getenv("FT_FA_FWD"); return e && std::string(e) == "v1"; }();
  if (variant == 0) variant = (force_v1 || S % 256 != 0) ? 1 : 2;
  TORCH_CHECK(variant >= 1 && variant <= 4, "flash_fwd: unknown variant");
  TORCH_CHECK(variant == 1 || S % 256 == 0, "flash_fwd: the two-tile kernel needs S % 256 == 0");
  if (variant != 1) {
    dim3 grid(B * nq, S / 256);
#define FT_FA_PP(DD, EE, OP)                                                                    \
    do {                                                                                       \
      const int smem = sizeof(fa2::Smem<DD>) + 1024;                                           \
      static unsigned long long cfg = 0;                                                       \
      smem_attr_once(fa2::flash_fwd_pp_kernel<DD, EE, OP>, smem, cfg);                         \
      fa2::flash_fwd_pp_kernel<DD, EE, OP><<<grid, fa2::NTHREADS, smem, st>>>(tm, p);         \
    } while (0)
    if (D == 128) {
      if (variant == 2) FT_FA_PP(128, false, false);
      else if (variant == 3) FT_FA_PP(128, false, true);
      else FT_FA_PP(128, true, true);
    } else {
      if (variant == 2) FT_FA_PP(64, false, false);
      else if (variant == 3) FT_FA_PP(64, false, true);
      else FT_FA_PP(64, true, true);
    }
#undef FT_FA_PP
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  dim3 grid(B * nq, S / 128);
  if (D == 128) {
    const int smem = sizeof(Smem<128>) + 1024;
    static unsigned long long cfg = 0;
    smem_attr_once(flash_fwd_kernel<128>, smem, cfg);
    flash_fwd_kernel<128><<<grid, NTHREADS, smem, st>>>(tm, p);
  } else {
    const int smem = sizeof(Smem<64>) + 1024;
    static unsigned long long cfg = 0;
    smem_attr_once(flash_fwd_kernel<64>, smem, cfg);
    flash_fwd_kernel<64><<<grid, NTHREADS, smem, st>>>(tm, p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void flash_fwd(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t S,
               int64_t nq, int64_t nkv, int64_t D, torch::Tensor& err) {
  flash_fwd_variant(qkv, o, lse, B, S, nq, nkv, D, err, 0);
}

}  // namespace ft
