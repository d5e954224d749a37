// Causal flash attention backward with grouped-query heads for sm_100a, on tcgen05.
//
// Inputs: the packed projection qkv [B*S, (nq + 2*nkv) * D], the forward output o and its
// gradient dout [B*S, nq*D] (bf16), and the forward LSE [B, nq, S] (fp32, natural log).
// Output: dqkv with the layout of qkv (bf16).
//
// Three launches:
//   1. pre:  delta = rowsum(dout * o) per (query, head) and lse2 = lse * log2(e);
//   2. main: one CTA per (batch, q-head, 128-key block j) iterates over the query blocks
//            i = j .. S/128-1 that see those keys (causal) and accumulates dK, dV in TMEM;
//            dQ of each (i, j) pair and the final dK, dV are added into one fp32 buffer
//            shaped like qkv with TMA bulk reductions (the reduction runs in L2, so the q
//            heads of a group and the key blocks of a query block need no atomics);
//   3. cvt:  fp32 buffer -> bf16 dqkv, applying the softmax scale to dQ and dK.
//
// Main kernel roles (320 threads):
//   warp 8     TMA producer: K_j, V_j once; per query block dO_i, then Q_i + lse2_i + delta_i
//   warp 9     MMA issuer (also owns TMEM):
//                dP^T = V dO_i^T     (TMEM dP, lanes = keys, columns = queries)
//                S^T  = K Q_i^T      (TMEM S)
//                dV  += P^T dO_i     (A = P^T from TMEM, packed bf16 over the S columns,
//                                    B = dO MN-major)
//                dK  += dS^T Q_i     (A = dS^T, B = Q MN-major)
//                dQ_i = dS K         (A = the same dS^T tile read MN-major, B = K MN-major),
//                                    written into the S columns after the dV product
//   warps 0-7  compute: two warps per TMEM lane quadrant (32 keys), each owning 64 of the
//              128 query columns: P^T = exp2(S^T * scale*log2e - lse2), causal mask on the
//              diagonal block, written back into TMEM as packed bf16; dS^T = P^T * (dP^T -
//              delta) to shared memory as a bf16 128-byte-swizzled tile; then dQ_i out of TMEM
//              into fp32 staging boxes and a bulk reduce-add to global memory; finally dV and
//              dK the same way.
// TMEM columns: S/dQ [0,128), dP [128,256), dV [256, 256+D), dK [256+D, 256+2D).
// All waits are bounded (2 s): on timeout the kernel records an error code and leaves.
//
// Reference: the backward is autograd through torch SDPA in the reference
// (femtotron/model/llama_partial_model.py:70 calls F.scaled_dot_product_attention).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tmap.h"

namespace ft {
namespace fab {

constexpr int BQ = 128;
constexpr int BKV = 128;
constexpr int NTHREADS = 320;
constexpr int PRODUCER_WARP = 8, MMA_WARP = 9;
constexpr float kLog2e = 1.4426950408889634f;

struct Params {
  int B, S, nq, nkv;
  const float* lse2;   // [B, nq, S], log2 domain
  const float* delta;  // [B, nq, S]
  float scale_log2;
  int nqb;
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
  // operand tiles: D/64 (or 2 for the P/dS tiles) chunks of [128 rows][64 bf16], 128B swizzle
  __nv_bfloat16 k[BKV * D];
  __nv_bfloat16 v[BKV * D];
  __nv_bfloat16 q[BQ * D];
  __nv_bfloat16 dout[BQ * D];
  __nv_bfloat16 p[BKV * BQ];   // fp32 staging boxes for dQ/dK/dV (P^T itself stays in TMEM)
  __nv_bfloat16 ds[BKV * BQ];  // dS^T (rows = keys); also fp32 staging
  float lse2[BQ];
  float delta[BQ];
  uint64_t kv_full, q_full, q_empty, do_full, do_empty;
  uint64_t s_full, dp_full, p_full, ds_full, dq_full, dq_read, dkv_full;
  uint32_t tmem_base;
};

// Write 32 fp32 values (one TMEM lane row) into a 32x32 fp32 box in the 128-byte swizzled
// layout the fp32 tensor map expects, then (lane 0) reduce-add the box into global memory.
__device__ __forceinline__ void stage_reduce(float* box, const uint32_t (&v)[32], int lane,
                                             const CUtensorMap* tm, int x, int y) {
  float* dst = box + lane * 32;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const int pos = (u ^ (lane & 7)) * 4;
    *reinterpret_cast<float4*>(dst + pos) =
        make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]),
                    __uint_as_float(v[4 * u + 2]), __uint_as_float(v[4 * u + 3]));
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_reduce_add_2d(tm, box, x, y);
    tma_store_commit();
  }
}

template <int D>
__global__ void __launch_bounds__(NTHREADS, 1)
    flash_bwd_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                     const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_acc, const Params p) {
  using Sm = Smem<D>;
  extern __shared__ uint8_t smem_raw[];
  Sm& s = *reinterpret_cast<Sm*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int bh = blockIdx.x;
  const int j = blockIdx.y;  // key block; low j (most query blocks) launches first
  const int b = bh / p.nq, h = bh % p.nq;
  const int g = h / (p.nq / p.nkv);
  const int niter = p.nqb - j;
  const int key_row0 = b * p.S + j * BKV;
  const int qcol = h * D, kcol = (p.nq + g) * D, vcol = (p.nq + p.nkv + g) * D;
  const int64_t stat0 = (static_cast<int64_t>(b) * p.nq + h) * p.S;
  constexpr int CH = D / 64;
  constexpr uint32_t TILE_BYTES = 128 * D * 2;

  if (threadIdx.x == 0) {
    mbar_init(&s.kv_full, 1);
    mbar_init(&s.q_full, 1);
    mbar_init(&s.q_empty, 1);
    mbar_init(&s.do_full, 1);
    mbar_init(&s.do_empty, 1);
    mbar_init(&s.s_full, 1);
    mbar_init(&s.dp_full, 1);
    mbar_init(&s.p_full, 8);
    mbar_init(&s.ds_full, 8);
    mbar_init(&s.dq_full, 1);
    mbar_init(&s.dq_read, 8);
    mbar_init(&s.dkv_full, 1);
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
  const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 256 + D;

  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      prefetch_tmap(&tm_qkv);
      prefetch_tmap(&tm_do);
      mbar_arrive_expect_tx(&s.kv_full, 2 * TILE_BYTES);
#pragma unroll
      for (int c = 0; c < CH; ++c) {
        tma_load_2d(s.k + c * 128 * 64, &tm_qkv, &s.kv_full, kcol + c * 64, key_row0);
        tma_load_2d(s.v + c * 128 * 64, &tm_qkv, &s.kv_full, vcol + c * 64, key_row0);
      }
      for (int it = 0; it < niter; ++it) {
        const int i = j + it;
        const int qrow = b * p.S + i * BQ;
        // dO_i may replace dO_{i-1} once dV_{i-1} is done
        if (it > 0 && !wait_b(&s.do_empty, (it - 1) & 1, p.err, 41)) break;
        mbar_arrive_expect_tx(&s.do_full, TILE_BYTES);
#pragma unroll
        for (int c = 0; c < CH; ++c) tma_load_2d(s.dout + c * 128 * 64, &tm_do, &s.do_full, qcol + c * 64, qrow);
        // Q_i (+ its LSE and delta rows) once dK_{i-1} is done (which also implies the compute
        // warps finished reading lse2/delta of block i-1)
        if (it > 0 && !wait_b(&s.q_empty, (it - 1) & 1, p.err, 42)) break;
        mbar_arrive_expect_tx(&s.q_full, TILE_BYTES + 2 * BQ * 4);
#pragma unroll
        for (int c = 0; c < CH; ++c) tma_load_2d(s.q + c * 128 * 64, &tm_qkv, &s.q_full, qcol + c * 64, qrow);
        bulk_load(s.lse2, p.lse2 + stat0 + i * BQ, BQ * 4, &s.q_full);
        bulk_load(s.delta, p.delta + stat0 + i * BQ, BQ * 4, &s.q_full);
      }
    }
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc_bf16(128, BQ, false, false);  // K-major x K-major
      constexpr uint32_t idKV = make_idesc_bf16(128, D, false, true);   // P^T/dS^T x (dO|Q)
      constexpr uint32_t idQ = make_idesc_bf16(128, D, true, true);     // dS (MN-major) x K
      const uint32_t ka = smem_u32(s.k), va = smem_u32(s.v), qa = smem_u32(s.q);
      const uint32_t doa = smem_u32(s.dout), dsa = smem_u32(s.ds);
      bool ok = wait_b(&s.kv_full, 0, p.err, 43);
      for (int it = 0; it < niter && ok; ++it) {
        const uint32_t par = it & 1;
        // dP^T = V dO^T  (TMEM dP is free: the compute warps signalled ds_full of it-1)
        if (!wait_b(&s.do_full, par, p.err, 44)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 128 * 128 + (kk & 3) * 32;
          mma_bf16(tdP, make_sw128_desc(va + off, 16, 1024), make_sw128_desc(doa + off, 16, 1024),
                   idS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.dp_full);
        // S^T = K Q^T into the S columns once dQ_{i-1} has been read out of them
        if (!wait_b(&s.q_full, par, p.err, 45)) { ok = false; break; }
        if (it > 0 && !wait_b(&s.dq_read, par ^ 1, p.err, 46)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 128 * 128 + (kk & 3) * 32;
          mma_bf16(tS, make_sw128_desc(ka + off, 16, 1024), make_sw128_desc(qa + off, 16, 1024),
                   idS, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.s_full);
        // dV += P^T dO, A = P^T from TMEM: packed bf16 pairs of queries 0..63 in S columns
        // 0..31 and of queries 64..127 in columns 64..95 (8 columns per 16 queries)
        if (!wait_b(&s.p_full, par, p.err, 47)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t at = tS + (kk >> 2) * 64 + (kk & 3) * 8;
          const uint64_t bd = make_sw128_desc(doa + kk * 2048, 128 * 128, 1024);
          mma_bf16_ts(tdV, at, bd, idKV, (it > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&s.do_empty);
        // dK += dS^T Q, then dQ = dS K into the S columns (the dV product above, which reads
        // P^T from those columns, was issued earlier, and tcgen05.mma operations of one
        // thread execute in order)
        if (!wait_b(&s.ds_full, par, p.err, 48)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint64_t ad = make_sw128_desc(dsa + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = make_sw128_desc(qa + kk * 2048, 128 * 128, 1024);
          mma_bf16(tdK, ad, bd, idKV, (it > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&s.q_empty);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk) {
          // A = dS: M = queries (contiguous, 2 chunks of 64), K = keys (rows, 16 per step)
          const uint64_t ad = make_sw128_desc(dsa + kk * 2048, 128 * 128, 1024);
          const uint64_t bd = make_sw128_desc(ka + kk * 2048, 128 * 128, 1024);
          mma_bf16(tS, ad, bd, idQ, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s.dq_full);
      }
      if (ok) mma_commit(&s.dkv_full);
    }
  } else {
    // ------------------------------------------------------------ compute warps 0..7
    const int quad = warp & 3, half = warp >> 2;
    const int r = quad * 32 + lane;  // key row within the block (TMEM lane)
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int col0 = half * (BQ / 2);  // this thread's 64 query columns
    // fp32 staging boxes of this warp: the 4 KB it owns in the staging tile and in the dS tile
    float* box0 = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.p) + half * 16384 + quad * 4096);
    float* box1 = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s.ds) + half * 16384 + quad * 4096);
    uint8_t* dsrow = reinterpret_cast<uint8_t*>(s.ds) + half * 128 * 128 + r * 128;
    bool ok = true;
    for (int it = 0; it < niter && ok; ++it) {
      const uint32_t par = it & 1;
      const int i = j + it;
      const bool diag = (it == 0);
      // ---- P^T
      if (!wait_b(&s.s_full, par, p.err, 49)) { ok = false; break; }
      tc_fence_after();
      float pv[BQ / 2];
      {
        uint32_t sv[BQ / 2];
        tmem_ld_32x32b_x32(tS + lane_off + col0, *reinterpret_cast<uint32_t(*)[32]>(sv));
        tmem_ld_32x32b_x32(tS + lane_off + col0 + 32, *reinterpret_cast<uint32_t(*)[32]>(sv + 32));
        tmem_wait_ld();
        const float4* L = reinterpret_cast<const float4*>(s.lse2 + col0);
#pragma unroll
        for (int c4 = 0; c4 < BQ / 8; ++c4) {
          const float4 l4 = L[c4];
          pv[4 * c4 + 0] = ex2_approx(fmaf(__uint_as_float(sv[4 * c4 + 0]), p.scale_log2, -l4.x));
          pv[4 * c4 + 1] = ex2_approx(fmaf(__uint_as_float(sv[4 * c4 + 1]), p.scale_log2, -l4.y));
          pv[4 * c4 + 2] = ex2_approx(fmaf(__uint_as_float(sv[4 * c4 + 2]), p.scale_log2, -l4.z));
          pv[4 * c4 + 3] = ex2_approx(fmaf(__uint_as_float(sv[4 * c4 + 3]), p.scale_log2, -l4.w));
        }
        if (diag) {  // query col0 + c sees key r only when col0 + c >= r
#pragma unroll
          for (int c = 0; c < BQ / 2; ++c)
            if (col0 + c < r) pv[c] = 0.f;
        }
      }
      // P^T as packed bf16 pairs into the first 32 of this warp's 64 S columns (all of which
      // this warp has read): the dV product takes it from TMEM
#pragma unroll
      for (int h16 = 0; h16 < 2; ++h16) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) pk[c] = pack_bf16x2(pv[32 * h16 + 2 * c], pv[32 * h16 + 2 * c + 1]);
        tmem_st_32x32b_x16(tS + lane_off + col0 + 16 * h16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full);
      // the staging boxes (inside the P and dS tiles) must have been read by the bulk
      // reductions of the previous block before they are overwritten
      if (it > 0) {
        if (lane == 0) tma_store_wait_read();
        __syncwarp();
      }
      // ---- dS^T = P^T * (dP^T - delta)
      if (!wait_b(&s.dp_full, par, p.err, 50)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int h32 = 0; h32 < 2; ++h32) {
        uint32_t dv[32];
        tmem_ld_32x32b_x32(tdP + lane_off + col0 + h32 * 32, dv);
        tmem_wait_ld();
        const float4* Dl = reinterpret_cast<const float4*>(s.delta + col0 + h32 * 32);
        float ds[32];
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 d4 = Dl[c4];
          ds[4 * c4 + 0] = pv[h32 * 32 + 4 * c4 + 0] * (__uint_as_float(dv[4 * c4 + 0]) - d4.x);
          ds[4 * c4 + 1] = pv[h32 * 32 + 4 * c4 + 1] * (__uint_as_float(dv[4 * c4 + 1]) - d4.y);
          ds[4 * c4 + 2] = pv[h32 * 32 + 4 * c4 + 2] * (__uint_as_float(dv[4 * c4 + 2]) - d4.z);
          ds[4 * c4 + 3] = pv[h32 * 32 + 4 * c4 + 3] * (__uint_as_float(dv[4 * c4 + 3]) - d4.w);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int pos = ((h32 * 4 + u) ^ (r & 7)) * 16;
          *reinterpret_cast<uint4*>(dsrow + pos) =
              make_uint4(pack_bf16x2(ds[8 * u], ds[8 * u + 1]), pack_bf16x2(ds[8 * u + 2], ds[8 * u + 3]),
                         pack_bf16x2(ds[8 * u + 4], ds[8 * u + 5]), pack_bf16x2(ds[8 * u + 6], ds[8 * u + 7]));
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.ds_full);
      // ---- dQ_i (rows = queries of block i) out of TMEM, reduce-added into the accumulator
      if (!wait_b(&s.dq_full, par, p.err, 51)) { ok = false; break; }
      tc_fence_after();
      const int qrow = b * p.S + i * BQ + quad * 32;
      if constexpr (D == 128) {
        uint32_t q0[32], q1[32];
        tmem_ld_32x32b_x32(tS + lane_off + half * 64, q0);
        tmem_ld_32x32b_x32(tS + lane_off + half * 64 + 32, q1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.dq_read);
        stage_reduce(box0, q0, lane, &tm_acc, qcol + half * 64, qrow);
        stage_reduce(box1, q1, lane, &tm_acc, qcol + half * 64 + 32, qrow);
      } else {
        uint32_t q0[32];
        tmem_ld_32x32b_x32(tS + lane_off + half * 32, q0);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.dq_read);
        stage_reduce(box0, q0, lane, &tm_acc, qcol + half * 32, qrow);
      }
    }
    // ---- dV, dK of this key block (rows = keys), D/2 columns per warp
    if (ok && wait_b(&s.dkv_full, 0, p.err, 52)) {
      tc_fence_after();
      if (lane == 0) tma_store_wait_read();
      __syncwarp();
#pragma unroll 1
      for (int t = 0; t < 2 * (D / 64); ++t) {
        const bool is_v = t < D / 64;
        const int cc = is_v ? t : t - D / 64;  // 32-column chunk within this warp's half
        const uint32_t src = (is_v ? tdV : tdK) + lane_off + half * (D / 2) + cc * 32;
        uint32_t v[32];
        tmem_ld_32x32b_x32(src, v);
        tmem_wait_ld();
        float* box = (t & 1) ? box1 : box0;
        if (t >= 2) {
          if (lane == 0) tma_store_wait_read_le1();
          __syncwarp();
        }
        stage_reduce(box, v, lane, &tm_acc, (is_v ? vcol : kcol) + half * (D / 2) + cc * 32,
                     key_row0 + quad * 32);
      }
    }
    if (lane == 0) tma_store_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b, h, s] = sum_d dout * o (fp32), lse2 = lse * log2(e); one warp per (token, head).
template <int D>
__global__ void flash_bwd_pre_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo,
                                     const __nv_bfloat16* __restrict__ dout, int64_t lddo,
                                     const float* __restrict__ lse, float* __restrict__ lse2,
                                     float* __restrict__ delta, int64_t rows, int S, int nq) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows * nq) return;
  const int64_t t = w / nq;
  const int h = static_cast<int>(w % nq);
  constexpr int E = D / 32;  // elements per lane (2 or 4)
  const __nv_bfloat16* orow = o + t * ldo + h * D + lane * E;
  const __nv_bfloat16* drow = dout + t * lddo + h * D + lane * E;
  float acc = 0.f;
  if constexpr (E == 4) {
    const uint2 a = *reinterpret_cast<const uint2*>(orow);
    const uint2 c = *reinterpret_cast<const uint2*>(drow);
    const float2 a0 = unpack_bf16x2(a.x), a1 = unpack_bf16x2(a.y);
    const float2 c0 = unpack_bf16x2(c.x), c1 = unpack_bf16x2(c.y);
    acc = a0.x * c0.x + a0.y * c0.y + a1.x * c1.x + a1.y * c1.y;
  } else {
    const float2 a0 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(orow));
    const float2 c0 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(drow));
    acc = a0.x * c0.x + a0.y * c0.y;
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const int64_t bb = t / S, ss = t % S;
    const int64_t idx = (bb * nq + h) * S + ss;
    delta[idx] = acc;
    lse2[idx] = lse[idx] * kLog2e;
  }
}

// dqkv[:, c] = bf16(acc[:, c] * (c < scaled_cols ? scale : 1)); 8 columns per thread.
__global__ void flash_bwd_cvt_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ out,
                                     int64_t rows, int64_t cols, int64_t ldo, int64_t scaled_cols,
                                     float scale) {
  const int64_t n8 = rows * (cols / 8);
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < n8;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = v / (cols / 8), c = (v % (cols / 8)) * 8;
    const float4* src = reinterpret_cast<const float4*>(acc + row * cols + c);
    const float4 a = src[0], bq = src[1];
    const float sc = c < scaled_cols ? scale : 1.f;
    *reinterpret_cast<uint4*>(out + row * ldo + c) =
        make_uint4(pack_bf16x2(a.x * sc, a.y * sc), pack_bf16x2(a.z * sc, a.w * sc),
                   pack_bf16x2(bq.x * sc, bq.y * sc), pack_bf16x2(bq.z * sc, bq.w * sc));
  }
}

template <int D>
void launch_main(const CUtensorMap& tq, const CUtensorMap& td, const CUtensorMap& ta, const Params& p,
                 dim3 grid, cudaStream_t st) {
  const int smem = sizeof(Smem<D>) + 1024;
  static unsigned long long cfg = 0;
  smem_attr_once(flash_bwd_kernel<D>, smem, cfg);
  flash_bwd_kernel<D><<<grid, NTHREADS, smem, st>>>(tq, td, ta, p);
}

}  // namespace fab

void flash_bwd(const torch::Tensor& qkv, const torch::Tensor& o, const torch::Tensor& dout,
               const torch::Tensor& lse, torch::Tensor& dqkv, int64_t B, int64_t S, int64_t nq,
               int64_t nkv, int64_t D, torch::Tensor& err) {
  using namespace fab;
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.stride(1) == 1);
  TORCH_CHECK(D == 64 || D == 128, "flash_bwd: head_dim 64 or 128");
  TORCH_CHECK(S % 128 == 0, "flash_bwd: sequence length must be a multiple of 128");
  TORCH_CHECK(nq % nkv == 0, "flash_bwd: q heads must be a multiple of kv heads");
  const int64_t W = (nq + 2 * nkv) * D;
  TORCH_CHECK(qkv.size(0) == B * S && qkv.size(1) >= W);
  TORCH_CHECK(o.scalar_type() == at::kBFloat16 && o.stride(1) == 1 && o.stride(0) % 8 == 0 &&
              o.size(0) == B * S && o.size(1) >= nq * D);
  TORCH_CHECK(dout.scalar_type() == at::kBFloat16 && dout.stride(1) == 1 && dout.stride(0) % 8 == 0 &&
              dout.size(0) == B * S && dout.size(1) >= nq * D);
  TORCH_CHECK(lse.is_contiguous() && lse.scalar_type() == at::kFloat && lse.numel() == B * nq * S);
  TORCH_CHECK(dqkv.scalar_type() == at::kBFloat16 && dqkv.stride(1) == 1 && dqkv.size(0) == B * S &&
              dqkv.size(1) == W && dqkv.stride(0) % 8 == 0);
  const c10::cuda::CUDAGuard g(qkv.device());
  auto st = at::cuda::getCurrentCUDAStream();
  auto f32 = qkv.options().dtype(at::kFloat);
  torch::Tensor acc = torch::zeros({B * S, W}, f32);
  torch::Tensor lse2 = torch::empty({B, nq, S}, f32);
  torch::Tensor delta = torch::empty({B, nq, S}, f32);
  {
    const int64_t warps = B * S * nq;
    const int blocks = static_cast<int>((warps + 7) / 8);
    if (D == 128)
      flash_bwd_pre_kernel<128><<<blocks, 256, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), o.stride(0),
          reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0), lse.data_ptr<float>(),
          lse2.data_ptr<float>(), delta.data_ptr<float>(), B * S, S, nq);
    else
      flash_bwd_pre_kernel<64><<<blocks, 256, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(o.data_ptr()), o.stride(0),
          reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()), dout.stride(0), lse.data_ptr<float>(),
          lse2.data_ptr<float>(), delta.data_ptr<float>(), B * S, S, nq);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
  CUtensorMap tq = make_tmap_2d(qkv.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, qkv.size(1),
                                qkv.size(0), qkv.stride(0), 64, 128, true);
  CUtensorMap td = make_tmap_2d(dout.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dout.size(1),
                                dout.size(0), dout.stride(0), 64, 128, true);
  CUtensorMap ta = make_tmap_2d(acc.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, W, B * S, W, 32, 32, true);
  Params p;
  p.B = B; p.S = S; p.nq = nq; p.nkv = nkv;
  p.lse2 = lse2.data_ptr<float>();
  p.delta = delta.data_ptr<float>();
  p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D))) * kLog2e;
  p.nqb = S / 128;
  p.err = err.data_ptr<int>();
  dim3 grid(B * nq, S / 128);
  if (D == 128)
    launch_main<128>(tq, td, ta, p, grid, st);
  else
    launch_main<64>(tq, td, ta, p, grid, st);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  {
    const int64_t n8 = B * S * (W / 8);
    int dev = qkv.get_device(), sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int blocks = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, sms * 8));
    flash_bwd_cvt_kernel<<<blocks, 256, 0, st>>>(acc.data_ptr<float>(),
                                                 reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr()), B * S, W,
                                                 dqkv.stride(0), (nq + nkv) * D,
                                                 static_cast<float>(1.0 / std::sqrt(static_cast<double>(D))));
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

}  // namespace ft
