// Persistent tcgen05 GEMM for sm_100a.
//
//   D[M,N] (op)= A[M,K] * B[N,K]^T      (fp32 accumulation in TMEM, bf16 operands)
//
// A and B may each be K-major (row-major with K contiguous) or MN-major (K rows, M/N
// contiguous), so one kernel covers the three linear-layer products:
//   forward  Y  = X  W^T : A = X  (K-major),  B = W  (K-major)
//   dgrad    dX = dY W   : A = dY (K-major),  B = W  (MN-major)
//   wgrad    dW = dY^T X : A = dY (MN-major), B = X  (MN-major)
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: one lane streams A/B k-blocks into a STAGES-deep smem ring.
//   warp 1      MMA issuer:   one lane issues tcgen05.mma (M=128, N=BN, K=16) into one of two
//                             TMEM accumulators and commits to mbarriers.
//   warp 2      TMEM allocator (512 columns = two BN<=256 fp32 accumulators).
//   warps 4..7  epilogue: tcgen05.ld of their 32 TMEM lanes, fused epilogue op, global store.
// The double-buffered accumulator lets the epilogue of tile i overlap the MMAs of tile i+1.
// No TMA multicast is used anywhere (each CTA loads its own tiles).
//
// Fused epilogues: plain bf16/fp32 store, in-place accumulation into an fp32 or bf16
// gradient buffer (wgrad of gradient accumulation), residual add (o_proj / down_proj), and
// SwiGLU (gate/up projection: the B tile pairs 128 gate rows with the matching 128 up rows).
//
// Every mbarrier wait is bounded by a wall-clock limit; on expiry the kernel records an error
// code in `err` and leaves its loops, so a bug cannot spin a GPU forever.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"
#include "tmap.h"

namespace ft {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one SW128 row
constexpr int NUM_THREADS = 256;
constexpr int EPI_WARP0 = 4;

enum EpiMode : int {
  EPI_STORE_BF16 = 0,   // D = acc (bf16)
  EPI_STORE_F32 = 1,    // D = acc (fp32)
  EPI_ACC_F32 = 2,      // D += acc (fp32)
  EPI_ACC_BF16 = 3,     // D += acc (bf16 storage, fp32 math)
  EPI_RESID_BF16 = 4,   // D = acc + R (bf16)
  EPI_SWIGLU_BF16 = 5,  // tile = [gate 128 | up 128]: D = silu(g)*u, and g,u stored to GU
  EPI_SCATTER_BF16 = 6, // D rows stored into their owner rank's buffer (scatter_base)
};

struct Params {
  int M, N, K;
  void* D;
  int64_t ldd;
  const __nv_bfloat16* R;  // residual (EPI_RESID_BF16)
  int64_t ldr;
  __nv_bfloat16* GU;       // gate/up pre-activations (EPI_SWIGLU_BF16): [M, gate_up_off + N]
  int64_t ldgu;
  int mode;
  int gate_up_off;         // EPI_SWIGLU_BF16: first row of the up block inside B
  int group_m;
  int* err;
  // Operand gate (fused all-gather -> GEMM): before loading a tile, the producer waits until
  // gate_flags[c] >= gate_epoch for every chunk c the tile's operand rows touch, where row r
  // of the gated operand lies in chunk (gate_off + r * gate_row_elems) / gate_chunk_elems.
  const int* gate_flags;
  int gate_op;             // 0 none, 1 gate A rows, 2 gate B rows (K-major operands only)
  int gate_epoch;
  int64_t gate_off, gate_row_elems, gate_chunk_elems;
  // SMs a gated launch leaves free for the kernels that release its gate (0: the default)
  int reserved_sms;
  // Row rotation of the tile order (a multiple of 256 rows; 0 = none): tiles are visited
  // starting at this output row, so a gated GEMM computes first on the rows that arrive first
  // (the local chunk of an all-gather, then the peers' chunks in the order they are pulled).
  int m_rot_rows;
  // Scatter epilogue (fused GEMM -> reduce-scatter): row r goes to owner o = r / scatter_rows,
  // stored at scatter_base[o] + (r - o * scatter_rows) * ldd (peer memory over NVLink).
  __nv_bfloat16* scatter_base[8];
  int scatter_rows;
};

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded mbarrier wait: about two seconds of wall clock, then record `code` and give up.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 128; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > 2000000000ull) {
      if (err) atomicCAS(err, 0, code);   // keep the first error (the root cause)
      return false;
    }
  }
}

// Fused all-gather gate: wait (bounded) for the chunks holding operand rows [r0, r1).
__device__ __forceinline__ bool gate_wait(const Params& p, int64_t r0, int64_t r1) {
  if (r1 <= r0) return true;
  const int64_t c0 = (p.gate_off + r0 * p.gate_row_elems) / p.gate_chunk_elems;
  const int64_t c1 = (p.gate_off + (r1 - 1) * p.gate_row_elems) / p.gate_chunk_elems;
  const uint64_t t0 = global_ns();
  for (int64_t c = c0; c <= c1; ++c) {
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p.gate_flags + c) : "memory");
      if (v - p.gate_epoch >= 0) break;
      if (global_ns() - t0 > 4000000000ull) {
        if (p.err) atomicCAS(p.err, 0, 40);
        return false;
      }
      __nanosleep(128);
    }
  }
  // data written by the copy engines is read next through the TMA (async) proxy
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// Row-tile index after the tile-order rotation of Params::m_rot_rows (tiles of tile_rows rows).
__device__ __forceinline__ int rotate_m(int tm, int tiles_m, int m_rot_rows, int tile_rows) {
  return m_rot_rows ? (tm + m_rot_rows / tile_rows) % tiles_m : tm;
}

// Grouped tile order: walk group_m row-tiles down a column before moving right, so one
// wave of CTAs touches few A row-panels and few B column-panels (L2 reuse).
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int group_m,
                                            int& tm, int& tn) {
  const int per_group = group_m * tiles_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gsize = min(tiles_m - first_m, group_m);
  const int r = t - g * per_group;
  tm = first_m + (r % gsize);
  tn = r / gsize;
}

template <int BN, int STAGES>
struct Smem {
  __nv_bfloat16 a[STAGES][BM * BK];
  __nv_bfloat16 b[STAGES][BN * BK];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
};

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v, int valid) {
  // valid: number of valid columns (multiple of 8) starting at dst.
  uint32_t pk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int j = 0; j < 4; ++j)
    if (j * 8 < valid) d4[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float* v, int valid) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 q = (j * 8 < valid) ? s4[j] : make_uint4(0, 0, 0, 0);
    float2 f;
    f = unpack_bf16x2(q.x); v[8 * j + 0] = f.x; v[8 * j + 1] = f.y;
    f = unpack_bf16x2(q.y); v[8 * j + 2] = f.x; v[8 * j + 3] = f.y;
    f = unpack_bf16x2(q.z); v[8 * j + 4] = f.x; v[8 * j + 5] = f.y;
    f = unpack_bf16x2(q.w); v[8 * j + 6] = f.x; v[8 * j + 7] = f.y;
  }
}

// Epilogue of one accumulator tile for the 32 rows of TMEM lane quadrant `q` (one row per
// thread): read fp32 accumulators 32 columns at a time and apply the fused op.
template <int BN>
__device__ __forceinline__ void epilogue_tile(const Params& p, uint32_t tmem_acc, int q, int lane,
                                              int row, int n0, bool swiglu) {
  const bool row_ok = row < p.M;
  const uint32_t tbase = tmem_acc + (static_cast<uint32_t>(q * 32) << 16);

      if (!swiglu) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld_32x32b_x32(tbase + c * 32, r);
          tmem_wait_ld();
          const int col0 = n0 + c * 32;
          const int valid = min(32, p.N - col0);
          if (row_ok && valid > 0) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            if (p.mode == EPI_STORE_BF16 || p.mode == EPI_RESID_BF16 || p.mode == EPI_ACC_BF16 ||
                p.mode == EPI_SCATTER_BF16) {
              __nv_bfloat16* d;
              if (p.mode == EPI_SCATTER_BF16) {
                const int owner = row / p.scatter_rows;
                if (!FT_DCHECK(owner < 8 && p.scatter_base[owner] != nullptr, p.err, 90)) continue;
                d = p.scatter_base[owner] + (int64_t)(row - owner * p.scatter_rows) * p.ldd + col0;
              } else {
                d = reinterpret_cast<__nv_bfloat16*>(p.D) + (int64_t)row * p.ldd + col0;
              }
              if (p.mode != EPI_STORE_BF16 && p.mode != EPI_SCATTER_BF16) {
                float o[32];
                if (p.mode == EPI_RESID_BF16)
                  load_bf16x32(p.R + (int64_t)row * p.ldr + col0, o, valid);
                else
                  load_bf16x32(d, o, valid);
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] += o[i];
              }
              store_bf16x32(d, v, valid);
            } else {
              float* d = reinterpret_cast<float*>(p.D) + (int64_t)row * p.ldd + col0;
              float4* d4 = reinterpret_cast<float4*>(d);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                if (j * 4 < valid) {
                  float4 x = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                  if (p.mode == EPI_ACC_F32) {
                    float4 o = d4[j];
                    x.x += o.x; x.y += o.y; x.z += o.z; x.w += o.w;
                  }
                  d4[j] = x;
                }
              }
            }
          }
        }
      } else {
        constexpr int HALF = BN / 2;
#pragma unroll 1
        for (int c = 0; c < HALF / 32; ++c) {
          uint32_t rg[32], ru[32];
          tmem_ld_32x32b_x32(tbase + c * 32, rg);
          tmem_ld_32x32b_x32(tbase + HALF + c * 32, ru);
          tmem_wait_ld();
          const int col0 = n0 + c * 32;
          const int valid = min(32, p.N - col0);
          if (row_ok && valid > 0) {
            float g[32], u[32], h[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              g[i] = __uint_as_float(rg[i]);
              u[i] = __uint_as_float(ru[i]);
              // Round the pre-activations to bf16 first so the forward matches what the
              // backward (which reads the stored bf16 g,u) differentiates.
              const float gb = __bfloat162float(__float2bfloat16_rn(g[i]));
              const float ub = __bfloat162float(__float2bfloat16_rn(u[i]));
              h[i] = gb / (1.0f + __expf(-gb)) * ub;
            }
            __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(p.D) + (int64_t)row * p.ldd + col0;
            store_bf16x32(d, h, valid);
            __nv_bfloat16* gu = p.GU + (int64_t)row * p.ldgu;
            store_bf16x32(gu + col0, g, valid);
            store_bf16x32(gu + p.gate_up_off + col0, u, valid);
          }
        }
      }
}

template <bool A_MN, bool B_MN, int BN, int STAGES>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                const Params p) {
  using S = Smem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  S& s = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool swiglu = (p.mode == EPI_SWIGLU_BF16);
  const int out_cols = swiglu ? (BN / 2) : BN;  // output columns per tile
  const int tiles_m = (p.M + BM - 1) / BM;
  const int tiles_n = (p.N + out_cols - 1) / out_cols;
  const int num_tiles = tiles_m * tiles_n;
  const int kblocks = (p.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 4);
    }
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc(&s.tmem_base, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
        tm = rotate_m(tm, tiles_m, p.m_rot_rows, BM);
        const int m0 = tm * BM;
        const int n0 = tn * out_cols;
        if (p.gate_op == 1 && !gate_wait(p, m0, min(m0 + BM, p.M))) { ok = false; break; }
        if (p.gate_op == 2 && !gate_wait(p, n0, min(n0 + BN, p.N))) { ok = false; break; }
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bar(&s.empty[stage], phase ^ 1, p.err, 1)) { ok = false; break; }
          mbar_arrive_expect_tx(&s.full[stage], (BM + BN) * BK * 2);
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d(s.a[stage], &tma_a, &s.full[stage], k0, m0);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_2d(s.a[stage] + j * 64 * BK, &tma_a, &s.full[stage], m0 + 64 * j, k0);
          }
          if (!B_MN) {
            if (swiglu) {
              tma_load_2d(s.b[stage], &tma_b, &s.full[stage], k0, n0);
              tma_load_2d(s.b[stage] + (BN / 2) * BK, &tma_b, &s.full[stage], k0,
                          p.gate_up_off + n0);
            } else {
              tma_load_2d(s.b[stage], &tma_b, &s.full[stage], k0, n0);
            }
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(s.b[stage] + j * 64 * BK, &tma_b, &s.full[stage], n0 + 64 * j, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        if (!wait_bar(&s.acc_empty[acc], acc_phase ^ 1, p.err, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * BN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bar(&s.full[stage], phase, p.err, 3)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(s.a[stage]);
          const uint32_t b_base = smem_u32(s.b[stage]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_sw128_desc(a_base + kk * 2048, 64 * BK * 2, 1024)
                                     : make_sw128_desc(a_base + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sw128_desc(b_base + kk * 2048, 64 * BK * 2, 1024)
                                     : make_sw128_desc(b_base + kk * 32, 16, 1024);
            mma_bf16(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&s.empty[stage]);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&s.acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------- Epilogue ----------------
    const int q = warp - EPI_WARP0;  // TMEM lane quadrant owned by this warp
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
      tm = rotate_m(tm, tiles_m, p.m_rot_rows, BM);
      const int m0 = tm * BM;
      const int n0 = tn * out_cols;
      if (!wait_bar(&s.acc_full[acc], acc_phase, p.err, 4)) break;
      tc_fence_after();
      epilogue_tile<BN>(p, tmem + acc * BN, q, lane, m0 + q * 32 + lane, n0, swiglu);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}


// ------------------------------------------------------------------------------------------
// 2-SM variant: a CTA pair (cluster of 2) computes a 256 x 256 tile with tcgen05.mma
// cta_group::2.  Each CTA stages its own 128 rows of A and its own 128-column half of B
// (loaded by itself, no multicast); the leader CTA issues the MMAs, whose operands come
// from both CTAs' shared memory at the same offsets, and each CTA's TMEM receives its 128
// accumulator rows.  Halving the B tile per CTA halves the operand bytes each SM reads per
// MMA, which is what lets the tensor cores run at full rate.
//   full[s]      leader only: both CTAs' TMA bytes complete on it (expect_tx = 2 stages)
//   empty[s]     both CTAs: the leader's commit multicasts to the pair when the stage is read
//   acc_full[a]  both CTAs: commit multicast when accumulator a is complete
//   acc_empty[a] leader only: 4 epilogue warps of each CTA arrive (8) when a is drained
// ------------------------------------------------------------------------------------------
constexpr int PAIR_BN = 256;

// fp32 epilogue through TMA: each warp moves its 32 accumulator rows 32 columns at a time
// from TMEM into a 32x32 fp32 staging box in shared memory (128-byte swizzled rows, so the
// row-per-lane writes hit distinct banks), then one lane issues a bulk tensor store or an
// in-L2 reduce-add of the box into D.  The SM never reads D back, and the writes are
// full-line, coalesced transfers.  Two staging boxes per warp alternate; a box is rewritten
// only after the bulk copy that read it has finished reading.
template <int PBN>
__device__ __forceinline__ void epilogue_tile_f32_tma(const Params& p, const CUtensorMap* tma_d,
                                                      float (*box)[32 * 32], uint32_t tmem_acc,
                                                      int q, int lane, int row0, int n0, bool add,
                                                      int& buf) {
  const uint32_t tbase = tmem_acc + (static_cast<uint32_t>(q * 32) << 16);
#pragma unroll 1
  for (int c = 0; c < PBN / 32; ++c) {
    const int col0 = n0 + c * 32;
    uint32_t r[32];
    tmem_ld_32x32b_x32(tbase + c * 32, r);
    tmem_wait_ld();
    if (col0 >= p.N) continue;  // uniform across the warp
    if (lane == 0) tma_store_wait_read_le1();  // box `buf` is free again
    __syncwarp();
    float* dst = box[buf] + lane * 32;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int pos = (j ^ (lane & 7)) * 4;
      *reinterpret_cast<float4*>(dst + pos) = make_float4(
          __uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
          __uint_as_float(r[4 * j + 3]));
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (add)
        tma_reduce_add_2d(tma_d, box[buf], col0, row0);
      else
        tma_store_2d(tma_d, box[buf], col0, row0);
      tma_store_commit();
    }
    buf ^= 1;
  }
}

template <int BN, int STAGES>
struct PairSmem {
  __nv_bfloat16 a[STAGES][128 * BK];
  __nv_bfloat16 b[STAGES][(BN / 2) * BK];
  float epi[4][2][32 * 32];  // per epilogue warp: two 32x32 fp32 staging boxes (SW128 layout)
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
};

template <bool A_MN, bool B_MN, int PBN, int STAGES>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                     const __grid_constant__ CUtensorMap tma_b,
                     const __grid_constant__ CUtensorMap tma_d, const Params p) {
  using S = PairSmem<PBN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  S& s = *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);
  const bool swiglu = (p.mode == EPI_SWIGLU_BF16);
  constexpr int HB = PBN / 2;  // B rows (N columns) staged per CTA
  const int out_cols = swiglu ? HB : PBN;
  const int tiles_m = (p.M + 255) / 256;
  const int tiles_n = (p.N + out_cols - 1) / out_cols;
  const int num_tiles = tiles_m * tiles_n;
  const int kblocks = (p.K + BK - 1) / BK;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.acc_full[i], 1);
      mbar_init(&s.acc_empty[i], 8);
    }
    fence_barrier_init();
  }
  if (warp == 2) {
    tmem_alloc_pair(&s.tmem_base, 512);
    tmem_relinquish_pair();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tma_a);
    prefetch_tmap(&tma_b);
  }
  tc_fence_before();
  cluster_sync();  // barrier inits and TMEM allocations visible across the pair
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        int tm, tn;
        tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
        tm = rotate_m(tm, tiles_m, p.m_rot_rows, 256);
        const int m0 = tm * 256 + static_cast<int>(rank) * 128;
        const int n0 = tn * out_cols;
        // K-major B rows held by this CTA (SwiGLU: leader = gate rows, peer = up rows)
        const int brow = swiglu ? (leader ? n0 : p.gate_up_off + n0) : n0 + static_cast<int>(rank) * HB;
        if (p.gate_op == 1 && !gate_wait(p, m0, min(m0 + 128, p.M))) { ok = false; break; }
        if (p.gate_op == 2 && !gate_wait(p, brow, brow + HB)) { ok = false; break; }
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bar(&s.empty[stage], phase ^ 1, p.err, 11)) { ok = false; break; }
          if (leader) mbar_arrive_expect_tx(&s.full[stage], 2 * (128 + HB) * BK * 2);
          const uint32_t fb = mapa_shared(smem_u32(&s.full[stage]), 0);
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d_pair(s.a[stage], &tma_a, fb, k0, m0);
          } else {
            tma_load_2d_pair(s.a[stage], &tma_a, fb, m0, k0);
            tma_load_2d_pair(s.a[stage] + 64 * BK, &tma_a, fb, m0 + 64, k0);
          }
          if (!B_MN) {
            tma_load_2d_pair(s.b[stage], &tma_b, fb, k0, brow);
          } else {
            const int ncol = n0 + static_cast<int>(rank) * HB;
#pragma unroll
            for (int j = 0; j < HB / 64; ++j)
              tma_load_2d_pair(s.b[stage] + j * 64 * BK, &tma_b, fb, ncol + 64 * j, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // Drain: wait until the leader's MMAs released every stage of this CTA, so no commit
      // arrival targets this CTA's shared memory after it exits.
      for (int i = 0; i < STAGES && ok; ++i) {
        if (!wait_bar(&s.empty[stage], phase ^ 1, p.err, 12)) break;
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader only) ----------------
    if (leader && elect_one()) {
      constexpr uint32_t idesc = make_idesc_bf16(256, PBN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        if (!wait_bar(&s.acc_empty[acc], acc_phase ^ 1, p.err, 13)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem + acc * PBN;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bar(&s.full[stage], phase, p.err, 14)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(s.a[stage]);
          const uint32_t b_base = smem_u32(s.b[stage]);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? make_sw128_desc(a_base + kk * 2048, 64 * BK * 2, 1024)
                                     : make_sw128_desc(a_base + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? make_sw128_desc(b_base + kk * 2048, 64 * BK * 2, 1024)
                                     : make_sw128_desc(b_base + kk * 32, 16, 1024);
            mma_bf16_pair(d_tmem, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit_pair_mc(&s.empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit_pair_mc(&s.acc_full[acc], 0x3);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // Drain: both accumulators released by both CTAs' epilogues (their remote arrivals
      // have landed) before teardown.
      for (int i = 0; i < 2 && ok; ++i) {
        if (!wait_bar(&s.acc_empty[acc], acc_phase ^ 1, p.err, 15)) break;
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------- Epilogue (both CTAs) ----------------
    const int q = warp - EPI_WARP0;
    const bool f32_out = (p.mode == EPI_ACC_F32 || p.mode == EPI_STORE_F32);
    int epi_buf = 0;
    if (f32_out && lane == 0) prefetch_tmap(&tma_d);
    const uint32_t acc_empty_leader0 = mapa_shared(smem_u32(&s.acc_empty[0]), 0);
    const uint32_t acc_empty_leader1 = mapa_shared(smem_u32(&s.acc_empty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair; t < num_tiles; t += npairs) {
      int tm, tn;
      tile_coords(t, tiles_m, tiles_n, p.group_m, tm, tn);
      tm = rotate_m(tm, tiles_m, p.m_rot_rows, 256);
      const int m0 = tm * 256 + static_cast<int>(rank) * 128;
      const int n0 = tn * out_cols;
      if (!wait_bar(&s.acc_full[acc], acc_phase, p.err, 16)) break;
      tc_fence_after();
      if (f32_out)
        epilogue_tile_f32_tma<PBN>(p, &tma_d, s.epi[q], tmem + acc * PBN, q, lane, m0 + q * 32, n0,
                                   p.mode == EPI_ACC_F32, epi_buf);
      else
        epilogue_tile<PBN>(p, tmem + acc * PBN, q, lane, m0 + q * 32 + lane, n0, swiglu);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? acc_empty_leader1 : acc_empty_leader0);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (f32_out && lane == 0) tma_store_wait_all();  // bulk reductions done before exit
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair is done with each other's shared memory and TMEM
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------------
// Host launcher
// ------------------------------------------------------------------------------------------
static int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

// A gated GEMM (fused all-gather) waits for chunks that other streams bring in: the pull
// kernel (tp_comm.cu, one CTA per SM) or copy engines after one-warp flag waits.  A
// persistent grid over every SM could leave those kernels no SM to run on while the GEMM waits
// for them, so gated launches leave SMs free: Params::reserved_sms, or GATE_RESERVED_SMS (the
// pull kernel's CTA count) when the caller gives none.
constexpr int GATE_RESERVED_SMS = 16;

static int usable_sms(const Params& p) {
  if (p.gate_op == 0) return num_sms();
  const int keep = p.reserved_sms > 0 ? p.reserved_sms : GATE_RESERVED_SMS;
  return std::max(2, num_sms() - keep);
}

template <bool A_MN, bool B_MN, int BN, int STAGES>
static void launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int num_tiles,
                   cudaStream_t stream) {
  auto kern = gemm_kernel<A_MN, B_MN, BN, STAGES>;
  const int smem = static_cast<int>(sizeof(Smem<BN, STAGES>)) + 1024;
  static unsigned long long configured = 0;  // per device, one mask per template instance
  smem_attr_once(kern, smem, configured);
  const int grid = std::max(1, std::min(num_tiles, usable_sms(p)));
  kern<<<grid, NUM_THREADS, smem, stream>>>(ta, tb, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <bool A_MN, bool B_MN, int PBN>
static void launch_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& td,
                        const Params& p, int num_tiles, cudaStream_t stream) {
  constexpr int STAGES = PBN == 256 ? 6 : 7;
  auto kern = gemm_pair_kernel<A_MN, B_MN, PBN, STAGES>;
  const int smem = static_cast<int>(sizeof(PairSmem<PBN, STAGES>)) + 1024;
  static unsigned long long configured = 0;  // per device, one mask per template instance
  smem_attr_once(kern, smem, configured);
  const int pairs = std::max(1, std::min(num_tiles, usable_sms(p) / 2));
  kern<<<2 * pairs, NUM_THREADS, smem, stream>>>(ta, tb, td, p);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <bool A_MN, bool B_MN>
static void dispatch_bn(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const Params& p,
                        int num_tiles, cudaStream_t stream) {
  if (bn == 256)
    launch<A_MN, B_MN, 256, 4>(ta, tb, p, num_tiles, stream);
  else
    launch<A_MN, B_MN, 128, 6>(ta, tb, p, num_tiles, stream);
}

// Pick BN: 256-wide tiles (better operand reuse per UMMA) unless N is small, measured
// faster or equal on every Llama-3-8B projection shape; FT_GEMM_BN=128|256 forces one.
static int choose_bn(int M, int N, bool swiglu) {
  if (swiglu) return 256;
  static int forced = [] {
    const char* e = getenv("FT_GEMM_BN");
    return e ? atoi(e) : 0;
  }();
  if (forced == 128 || forced == 256) return forced;
  (void)M;
  return N > 128 ? 256 : 128;
}

}  // namespace gemm

int64_t gate_reserved_sms() { return gemm::GATE_RESERVED_SMS; }

struct GateScatter {
  int64_t gate_flags = 0;
  int gate_op = 0;
  int gate_epoch = 0;
  int64_t gate_off = 0, gate_row_elems = 1, gate_chunk_elems = 1;
  std::vector<int64_t> scatter_ptrs;
  int scatter_rows = 0;
  int64_t m_rot_rows = 0;
  int reserved_sms = 0;
};

void gemm_tc_impl(const torch::Tensor& A, const torch::Tensor& B, torch::Tensor& D, bool a_mn,
                  bool b_mn, int64_t mode, const c10::optional<torch::Tensor>& R,
                  const c10::optional<torch::Tensor>& GU, int64_t gate_up_off, torch::Tensor& err,
                  const GateScatter& gs);

// A: [M,K] (a_mn=false) or [K,M] (a_mn=true); B: [N,K] (b_mn=false) or [K,N] (b_mn=true).
// D: [M,N] bf16 or fp32 per `mode`.  All operands row-major with unit inner stride.
void gemm_tc(const torch::Tensor& A, const torch::Tensor& B, torch::Tensor& D, bool a_mn,
             bool b_mn, int64_t mode, const c10::optional<torch::Tensor>& R,
             const c10::optional<torch::Tensor>& GU, int64_t gate_up_off, torch::Tensor& err) {
  gemm_tc_impl(A, B, D, a_mn, b_mn, mode, R, GU, gate_up_off, err, GateScatter());
}

// Fused-communication GEMM: K-major operands, optional operand gate and scatter epilogue.
//   gate_op 1/2 gates A/B rows on int32 flags at `gate_flags` (device address);
//   mode 6 stores row r of D into scatter_ptrs[r / scatter_rows] (row stride D.stride(0));
//   m_rot_rows (a multiple of 256, or 0) starts the tile order at that output row;
//   reserved_sms (> 0) is how many SMs a gated launch leaves to the streams releasing it.
void gemm_tc_fused(const torch::Tensor& A, const torch::Tensor& B, torch::Tensor& D, bool a_mn,
                   bool b_mn, int64_t mode,
                   const c10::optional<torch::Tensor>& R, const c10::optional<torch::Tensor>& GU,
                   int64_t gate_up_off, torch::Tensor& err, int64_t gate_flags, int64_t gate_op,
                   int64_t gate_epoch, int64_t gate_off, int64_t gate_row_elems,
                   int64_t gate_chunk_elems, const std::vector<int64_t>& scatter_ptrs,
                   int64_t scatter_rows, int64_t m_rot_rows, int64_t reserved_sms) {
  GateScatter gs;
  gs.gate_flags = gate_flags;
  gs.gate_op = static_cast<int>(gate_op);
  gs.gate_epoch = static_cast<int>(gate_epoch);
  gs.gate_off = gate_off;
  gs.gate_row_elems = std::max<int64_t>(1, gate_row_elems);
  gs.gate_chunk_elems = std::max<int64_t>(1, gate_chunk_elems);
  gs.scatter_ptrs = scatter_ptrs;
  gs.scatter_rows = static_cast<int>(scatter_rows);
  gs.m_rot_rows = m_rot_rows;
  gs.reserved_sms = static_cast<int>(std::max<int64_t>(0, reserved_sms));
  TORCH_CHECK(scatter_ptrs.size() <= 8, "gemm_tc_fused: at most 8 scatter owners");
  if (mode == 6) TORCH_CHECK(scatter_rows > 0 && !scatter_ptrs.empty(), "gemm_tc_fused: scatter needs owners");
  TORCH_CHECK(gs.gate_op == 0 || (gs.gate_op == 1 && !a_mn) || (gs.gate_op == 2 && !b_mn),
              "gemm_tc_fused: only K-major operands can be gated");
  gemm_tc_impl(A, B, D, a_mn, b_mn, mode, R, GU, gate_up_off, err, gs);
}

void gemm_tc_impl(const torch::Tensor& A, const torch::Tensor& B, torch::Tensor& D, bool a_mn,
                  bool b_mn, int64_t mode, const c10::optional<torch::Tensor>& R,
                  const c10::optional<torch::Tensor>& GU, int64_t gate_up_off, torch::Tensor& err,
                  const GateScatter& gs) {
  using namespace gemm;
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && D.is_cuda(), "gemm_tc: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16,
              "gemm_tc: bf16 operands required");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && D.dim() == 2, "gemm_tc: 2-D operands required");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1 && (mode == 6 || D.stride(1) == 1),
              "gemm_tc: unit inner stride required");
  const int M = a_mn ? A.size(1) : A.size(0);
  const int K = a_mn ? A.size(0) : A.size(1);
  const bool swiglu = (mode == EPI_SWIGLU_BF16);
  const int N = D.size(1);
  const int Kb = b_mn ? B.size(0) : B.size(1);
  TORCH_CHECK(K == Kb, "gemm_tc: K mismatch ", K, " vs ", Kb);
  TORCH_CHECK(D.size(0) == M, "gemm_tc: D rows mismatch");
  const bool scatter = (mode == 6);
  if (swiglu) {
    TORCH_CHECK(!b_mn, "gemm_tc: swiglu epilogue needs a K-major B");
    TORCH_CHECK(B.size(0) >= gate_up_off + N, "gemm_tc: swiglu B too small");
    TORCH_CHECK(GU.has_value() && GU->size(0) == M && GU->size(1) >= gate_up_off + N,
                "gemm_tc: swiglu needs GU [M, gate_up_off+N]");
    TORCH_CHECK(N % 8 == 0 && gate_up_off % 8 == 0, "gemm_tc: swiglu sizes must be multiples of 8");
  } else {
    const int Nb = b_mn ? B.size(1) : B.size(0);
    TORCH_CHECK(Nb == N, "gemm_tc: N mismatch ", Nb, " vs ", N);
  }
  TORCH_CHECK(N % 8 == 0, "gemm_tc: N must be a multiple of 8");
  const bool out_f32 = (mode == EPI_STORE_F32 || mode == EPI_ACC_F32);
  TORCH_CHECK(D.scalar_type() == (out_f32 ? at::kFloat : at::kBFloat16), "gemm_tc: D dtype");
  if (!scatter)
    TORCH_CHECK(D.stride(0) % (out_f32 ? 4 : 8) == 0 &&
                    reinterpret_cast<uintptr_t>(D.data_ptr()) % 16 == 0,
                "gemm_tc: D must be 16-byte aligned with an aligned row stride");
  if (mode == EPI_RESID_BF16) {
    TORCH_CHECK(R.has_value() && R->scalar_type() == at::kBFloat16 && R->size(0) == M &&
                    R->size(1) == N && R->stride(1) == 1 && R->stride(0) % 8 == 0,
                "gemm_tc: bad residual");
  }
  const c10::cuda::CUDAGuard guard(A.device());
  auto stream = at::cuda::getCurrentCUDAStream();

  static const int pair_mode = [] {
    const char* e = getenv("FT_GEMM_PAIR");
    return e ? atoi(e) : 1;
  }();
  const bool use_pair = pair_mode != 0 && M > 128 && (swiglu || N > 128);
  // Pair tile width: 256 (best operand reuse) unless 128-wide tiles fill the last wave of
  // CTA pairs enough better.  Cost model: waves x (tile width x k-blocks + a fixed per-tile
  // pipeline fill/drain worth 8 k-blocks of a 256-wide tile), 5% extra for the narrow tile.
  int pbn = 256;
  if (use_pair && !swiglu) {
    const long pairs = std::max(1, num_sms() / 2);
    const long tm = (M + 255) / 256;
    const long kb = (K + BK - 1) / BK;
    const long c256 = (tm * ((N + 255) / 256) + pairs - 1) / pairs * (256 * kb + 2048);
    const long c128 = (tm * ((N + 127) / 128) + pairs - 1) / pairs * (128 * kb + 2048);
    if (c128 * 105 < c256 * 100) pbn = 128;
    if (pair_mode == 2) pbn = 256;
    if (pair_mode == 3) pbn = 128;
  }
  const int bn = use_pair ? pbn : choose_bn(M, N, swiglu);
  const auto BF16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const int a_rows = use_pair ? 128 : BM;            // rows of A staged per CTA
  const int b_rows = use_pair ? bn / 2 : (swiglu ? 128 : bn);  // K-major B rows per TMA box
  CUtensorMap ta = a_mn ? make_tmap_2d(A.data_ptr(), BF16, 2, M, K, A.stride(0), 64, 64, true)
                        : make_tmap_2d(A.data_ptr(), BF16, 2, K, M, A.stride(0), 64, a_rows, true);
  CUtensorMap tb;
  if (b_mn)
    tb = make_tmap_2d(B.data_ptr(), BF16, 2, B.size(1), K, B.stride(0), 64, 64, true);
  else
    tb = make_tmap_2d(B.data_ptr(), BF16, 2, K, B.size(0), B.stride(0), 64, b_rows, true);

  Params p;
  p.M = M; p.N = N; p.K = K;
  p.D = scatter ? nullptr : D.data_ptr();
  p.ldd = scatter ? N : D.stride(0);
  p.R = R.has_value() ? reinterpret_cast<const __nv_bfloat16*>(R->data_ptr()) : nullptr;
  p.ldr = R.has_value() ? R->stride(0) : 0;
  p.GU = GU.has_value() ? reinterpret_cast<__nv_bfloat16*>(GU->data_ptr()) : nullptr;
  p.ldgu = GU.has_value() ? GU->stride(0) : 0;
  p.mode = static_cast<int>(mode);
  p.gate_up_off = static_cast<int>(gate_up_off);
  p.group_m = 8;
  p.err = err.data_ptr<int>();
  p.gate_flags = reinterpret_cast<const int*>(gs.gate_flags);
  p.gate_op = gs.gate_op;
  p.gate_epoch = gs.gate_epoch;
  p.gate_off = gs.gate_off;
  p.gate_row_elems = gs.gate_row_elems;
  p.gate_chunk_elems = gs.gate_chunk_elems;
  // rotation in whole 256-row tiles (both the 128-row and the paired 256-row tilings)
  p.reserved_sms = gs.reserved_sms;
  p.m_rot_rows = (gs.m_rot_rows > 0 && gs.m_rot_rows % 256 == 0 && gs.m_rot_rows < M) ? gs.m_rot_rows : 0;
  for (int i = 0; i < 8; ++i)
    p.scatter_base[i] = i < static_cast<int>(gs.scatter_ptrs.size())
                            ? reinterpret_cast<__nv_bfloat16*>(gs.scatter_ptrs[i])
                            : nullptr;
  p.scatter_rows = gs.scatter_rows;

  const int out_cols = swiglu ? bn / 2 : bn;
  if (use_pair) {
    // fp32 output: TMA store / reduce-add map over D, 32x32 boxes with 128-byte swizzle
    CUtensorMap td = out_f32 ? make_tmap_2d(D.data_ptr(), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, M,
                                            D.stride(0), 32, 32, true)
                             : ta;  // unused for bf16 outputs
    const int pair_tiles = ((M + 255) / 256) * ((N + out_cols - 1) / out_cols);  // out_cols = bn (or bn/2)
    if (!a_mn && !b_mn) (bn == 256 ? launch_pair<false, false, 256>(ta, tb, td, p, pair_tiles, stream) : launch_pair<false, false, 128>(ta, tb, td, p, pair_tiles, stream));
    else if (!a_mn && b_mn) (bn == 256 ? launch_pair<false, true, 256>(ta, tb, td, p, pair_tiles, stream) : launch_pair<false, true, 128>(ta, tb, td, p, pair_tiles, stream));
    else if (a_mn && b_mn) (bn == 256 ? launch_pair<true, true, 256>(ta, tb, td, p, pair_tiles, stream) : launch_pair<true, true, 128>(ta, tb, td, p, pair_tiles, stream));
    else (bn == 256 ? launch_pair<true, false, 256>(ta, tb, td, p, pair_tiles, stream) : launch_pair<true, false, 128>(ta, tb, td, p, pair_tiles, stream));
    return;
  }
  const int num_tiles = ((M + BM - 1) / BM) * ((N + out_cols - 1) / out_cols);
  if (!a_mn && !b_mn) dispatch_bn<false, false>(bn, ta, tb, p, num_tiles, stream);
  else if (!a_mn && b_mn) dispatch_bn<false, true>(bn, ta, tb, p, num_tiles, stream);
  else if (a_mn && b_mn) dispatch_bn<true, true>(bn, ta, tb, p, num_tiles, stream);
  else dispatch_bn<true, false>(bn, ta, tb, p, num_tiles, stream);
}

}  // namespace ft
