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

void flash_fwd(const torch::Tensor& qkv, torch::Tensor& o, torch::Tensor& lse, int64_t B, int64_t S,
               int64_t nq, int64_t nkv, int64_t D, torch::Tensor& err) {
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
  dim3 grid(B * nq, S / 128);
  auto st = at::cuda::getCurrentCUDAStream();
  if (D == 128) {
    const int smem = sizeof(Smem<128>) + 1024;
    static bool cfg = false;
    if (!cfg) { cudaFuncSetAttribute(flash_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); cfg = true; }
    flash_fwd_kernel<128><<<grid, NTHREADS, smem, st>>>(tm, p);
  } else {
    const int smem = sizeof(Smem<64>) + 1024;
    static bool cfg = false;
    if (!cfg) { cudaFuncSetAttribute(flash_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); cfg = true; }
    flash_fwd_kernel<64><<<grid, NTHREADS, smem, st>>>(tm, p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace ft
