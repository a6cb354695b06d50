// gemm_sm100.cu -- persistent bf16 tensor-core GEMM for sm_100a.
//
// C[M,N] = op(A) @ op(B)^T with fp32 accumulation in TMEM.
//   * TMA (cp.async.bulk.tensor, 128-byte swizzle) stages 64-deep K slices of
//     A and B through a shared-memory ring;
//   * one thread issues tcgen05.mma (K=16 per instruction) into one of two
//     fp32 TMEM accumulators of 128 lanes x 256 columns (all 512 TMEM
//     columns), so the epilogue of tile i overlaps the main loop of tile i+1;
//   * eight epilogue warps read the accumulator with tcgen05.ld (each warp
//     owns one 32-lane TMEM quadrant and one 128-column half);
//   * persistent scheduling: each CTA (or CTA pair) walks the tile list.
// Two tile shapes share one kernel body:
//   CG = 1: one CTA computes a 128 x 256 tile (A 16 KB + B 32 KB per stage,
//           4 stages);
//   CG = 2: a CTA pair (cluster of 2, tcgen05 cta_group::2) computes a
//           256 x 256 tile: each CTA stages its 128 rows of A and half of the
//           256 rows of B (16 KB + 16 KB per stage, 6 stages), the leader
//           issues M=256 MMAs that read both CTAs' shared memory, and each
//           CTA's TMEM receives its 128 rows. Per CTA this halves the B
//           traffic into shared memory for the same math.
// Operands may be K-major ([rows, K] row-major) or MN-major ([K, rows]),
// which covers the three GEMMs of the distillation loss without transposes:
//   logits = h @ W^T      (A K-major, B K-major)
//   grad_h = dlogits @ W  (A K-major, B MN-major)
//   grad_W = dlogits^T @ h (A MN-major, B MN-major)
// Epilogues: plain scaled store (or TMA reduce-add), or the logits epilogue
// that writes fp32 logits and per-(row, 128-column part) online-softmax
// statistics (max, sum exp(x-m), sum exp((x-m)/T), sum x) from the fp32
// accumulators, so the loss needs no separate reduction pass over the logits.
// L2 policies: the operand that is small and reused by every tile is loaded
// evict-last, large streamed outputs are stored evict-first.
//
// No TMA load uses cluster multicast (the same kernels serve multi-GPU runs);
// the CTA pair's loads each land in their own CTA.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "fastmath.cuh"
#include "kernels.h"
#include "ptx.cuh"

namespace orda {

namespace {

constexpr int BN = 256;  // tile columns (N)
constexpr int BK = 64;   // K slice per stage (128 bytes of bf16)
constexpr int NUM_THREADS = 384;  // warp 0 TMA, 1 MMA, 2 TMEM, 3 idle, 4..11 epilogue
constexpr int EPI_WARP0 = 4;
constexpr int NUM_EPI_WARPS = 8;
constexpr int TMEM_COLS = 512;
// Per epilogue warp: one 32 x 32 fp32 output chunk staged for a TMA store.
constexpr int OUT_STAGE_BYTES = 32 * 32 * 4;
constexpr int OUT_BYTES = NUM_EPI_WARPS * OUT_STAGE_BYTES;  // 32 KB
constexpr float LOG2E = 1.4426950408889634f;

// WIDE (CTA pairs only): a 256 x 512 tile per pair, two N = 256 MMAs per K
// slice sharing the A stage, one accumulator filling all 512 TMEM columns.
// A CTA then stages 48 KB per K slice for 1024 MMA cycles instead of 32 KB
// for 512: a quarter fewer L2->SM bytes per FLOP and 3 slices (3072 cycles)
// of loads in flight instead of 5 x 512 = 2560 cycles. The single
// accumulator leaves the epilogue exposed once per tile, so it suits GEMMs
// with a long K loop per tile.
template <int CG, bool WIDE = false>
struct TileCfg {
  static_assert(!WIDE || CG == 2, "wide tiles are CTA-pair tiles");
  static constexpr int NW = WIDE ? 2 : 1;     // N = 256 MMAs per K slice
  static constexpr int TILE_M = 128 * CG;     // rows of C per tile
  static constexpr int TILE_N = BN * NW;      // columns of C per tile
  static constexpr int NACC = WIDE ? 1 : 2;   // TMEM accumulators
  static constexpr int B_PART = BN / CG;      // B rows one CTA stages per MMA
  static constexpr int B_ROWS = B_PART * NW;  // B rows staged by one CTA
  static constexpr int B_PART_BYTES = B_PART * BK * 2;
  static constexpr int A_STAGE = 128 * BK * 2;
  static constexpr int B_STAGE = B_ROWS * BK * 2;
  static constexpr int STAGE = A_STAGE + B_STAGE;
  static constexpr int STAGES = CG == 2 ? (WIDE ? 4 : 6) : 4;
  static constexpr int SMEM = STAGES * STAGE + OUT_BYTES + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(SMEM <= 232448, "shared memory over the sm_100 opt-in limit");
  static_assert((2 * STAGES + 5) * 8 + 4 <= 256, "barrier area");
};

struct KParams {
  int M, N;
  int m_blocks, n_blocks, num_tiles;  // m_blocks in units of TILE_M
  int raster_n_fastest;
  int group_m;     // M-fastest raster: tiles walk groups of group_m M blocks
  int nseg;
  int seg_kblocks[2];
  int* status;
  int tma_store;   // output written through the staging buffers + TMA
  int tma_reduce;  // TMA reduce-add into the output (beta == 1)
  int pol_a, pol_b, pol_c;  // L2 policy kinds (0 normal, 1 evict-first, 2 evict-last)
  int spare_sms;            // host side: SMs the persistent grid leaves free
  // Work items: tiles [0, full_tiles) over the whole K; then the rem_tiles
  // tiles of the last partial wave, each split into nsplit (1 or 2) K
  // halves whose partial sums are reduce-added into a zeroed output. An
  // unsplit tile sums K in one order whatever the tile shape; a split tile
  // sums each half in that order and adds the two.
  int full_tiles, rem_tiles, nsplit, num_items;
  int allow_split;  // host side: the output may take split tiles (plain TMA store, one K segment)
  EpiArgs e;
};

// Work item -> tile and its K-block range [kb0, kb1) (single K segment when
// split; otherwise kb0 = 0, kb1 = -1 meaning every segment in full).
__device__ __forceinline__ int work_item(const KParams& p, int w, int& kb0, int& kb1) {
  if (w < p.full_tiles) {
    kb0 = 0;
    kb1 = -1;
    return w;
  }
  const int j = w - p.full_tiles;
  const int part = j / p.rem_tiles;
  const int kb = p.seg_kblocks[0];
  kb0 = static_cast<int>(static_cast<long long>(kb) * part / p.nsplit);
  kb1 = static_cast<int>(static_cast<long long>(kb) * (part + 1) / p.nsplit);
  return p.full_tiles + j % p.rem_tiles;
}

// Tile index -> (M block, N block). N-fastest: the N blocks of one M block
// are consecutive. Otherwise M-fastest inside groups of group_m M blocks, so
// a wave of tiles shares a few B tiles and a bounded slab of A.
__device__ __forceinline__ void tile_coords(const KParams& p, int tile, int& mb, int& nb) {
  if (p.raster_n_fastest) {
    nb = tile % p.n_blocks;
    mb = tile / p.n_blocks;
  } else {
    const int per_group = p.group_m * p.n_blocks;
    const int g = tile / per_group;
    const int first_m = g * p.group_m;
    const int gm = min(p.group_m, p.m_blocks - first_m);
    const int r = tile - g * per_group;
    mb = first_m + r % gm;
    nb = r / gm;
  }
}

// ------------------------------------------------------------- epilogues

// Plain store: dst = alpha * acc (+ beta * dst).
__device__ __forceinline__ void epi_store_chunk(const KParams& p, long long grow, int col0, int nvalid,
                                                const uint32_t (&r)[32], float alpha) {
  const EpiArgs& e = p.e;
  float* dst;
  if (grow < e.split_row) dst = e.out0 + grow * e.ld0 + col0;
  else dst = e.out1 + (grow - e.split_row) * e.ld1 + col0;
  const bool vec = nvalid == 32 && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0);
  if (vec) {
#pragma unroll
    for (int j = 0; j < 32; j += 4) {
      float4 o;
      o.x = alpha * __uint_as_float(r[j + 0]);
      o.y = alpha * __uint_as_float(r[j + 1]);
      o.z = alpha * __uint_as_float(r[j + 2]);
      o.w = alpha * __uint_as_float(r[j + 3]);
      if (e.beta != 0.0f) {
        float4 old = *reinterpret_cast<const float4*>(dst + j);
        o.x += e.beta * old.x;
        o.y += e.beta * old.y;
        o.z += e.beta * old.z;
        o.w += e.beta * old.w;
      }
      *reinterpret_cast<float4*>(dst + j) = o;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (j < nvalid) {
        float o = alpha * __uint_as_float(r[j]);
        if (e.beta != 0.0f) o += e.beta * dst[j];
        dst[j] = o;
      }
    }
  }
}

struct OwnStats {
  float m, d1, dT, sx;
};

// e^x as 2^(x * log2 e) with the PTX ex2.approx.ftz.f32 instruction (one
// MUFU op); statistics sums of up to 128 terms tolerate its ~2^-22 relative
// error (checked against the f64 oracle by the parity tests).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max32(const float (&v)[32]) {
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) m[k] = fmaxf(fmaxf(v[4 * k], v[4 * k + 1]), fmaxf(v[4 * k + 2], v[4 * k + 3]));
#pragma unroll
  for (int k = 0; k < 4; ++k) m[k] = fmaxf(m[k], m[k + 4]);
  return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
}

// Online-softmax statistics of one 32-column chunk of one row. FULL: all 32
// columns valid (no per-element masking). POLY (Fast profile): one column in
// four of the tempered sum takes its exp2 from the FMA pipe (exp2_fma). With
// two exp2 and about eight other instructions per element the SFU (16 per
// SM-cycle) bounds this code; the ten-instruction polynomial on a quarter of
// one of the sums balances the SFU against the issue slots.
template <bool FULL, bool OWN_DT, bool POLY>
__device__ __forceinline__ void logits_chunk(const EpiArgs& e, long long grow, bool row_ok, int col0, int nvalid,
                                             const uint32_t (&r)[32], OwnStats& os) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  const float lt = LOG2E * e.inv_t;
  float vm[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) vm[j] = (FULL || j < nvalid) ? v[j] : -INFINITY;
  const float m_new = fmaxf(os.m, max32(vm));
  const float dm = os.m - m_new;  // -inf on the first chunk: factors 0
  os.d1 *= fast_exp2(dm * LOG2E);
  if (OWN_DT) os.dT *= fast_exp2(dm * lt);
  os.m = m_new;
  float a1[4] = {0.f, 0.f, 0.f, 0.f}, aT[4] = {0.f, 0.f, 0.f, 0.f}, ax[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (FULL || j < nvalid) {
      const float u = v[j] - m_new;
      a1[j & 3] += fast_exp2(u * LOG2E);
      if (OWN_DT) aT[j & 3] += (POLY && (j & 3) == 3) ? exp2_fma(u * lt) : fast_exp2(u * lt);
      ax[j & 3] += v[j];
    }
  }
  os.d1 += (a1[0] + a1[1]) + (a1[2] + a1[3]);
  if (OWN_DT) os.dT += (aT[0] + aT[1]) + (aT[2] + aT[3]);
  os.sx += (ax[0] + ax[1]) + (ax[2] + ax[3]);
}

template <bool OWN_DT, bool POLY>
__device__ __forceinline__ void logits_chunk_any(const EpiArgs& e, long long grow, bool row_ok, int col0, int N,
                                                 const uint32_t (&r)[32], OwnStats& os) {
  const int nvalid = N - col0;
  if (nvalid >= 32) logits_chunk<true, OWN_DT, POLY>(e, grow, row_ok, col0, 32, r, os);
  else if (nvalid > 0) logits_chunk<false, OWN_DT, POLY>(e, grow, row_ok, col0, nvalid, r, os);
}

// Two fp32 accumulator values as an fp16 pair (round to nearest, saturated to
// the largest finite fp16, so no logit becomes infinite); the first value in
// the low half (the lower address).
__device__ __forceinline__ uint32_t pack_f16x2_sat(uint32_t a, uint32_t b) {
  const float fa = fminf(fmaxf(__uint_as_float(a), -65504.0f), 65504.0f);
  const float fb = fminf(fmaxf(__uint_as_float(b), -65504.0f), 65504.0f);
  const __half2 h = __floats2half2_rn(fa, fb);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Writes the warp's 32 x 32 fp32 chunk (row `lane` = this thread's values,
// times alpha) to its staging buffer in the 128-byte-swizzled layout of the
// output tensor map, then one lane issues the TMA store (or reduce-add). The
// buffer is reused only after the previous store has read it.
__device__ __forceinline__ void stage_and_store(uint8_t* buf, int lane, const uint32_t (&r)[32], float alpha,
                                                const CUtensorMap* map, int x, int y, bool reduce,
                                                uint64_t policy) {
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float4 q = make_float4(alpha * __uint_as_float(r[4 * c]), alpha * __uint_as_float(r[4 * c + 1]),
                                 alpha * __uint_as_float(r[4 * c + 2]), alpha * __uint_as_float(r[4 * c + 3]));
    *reinterpret_cast<float4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) = q;
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (reduce) tma_reduce_add_2d_hint(map, buf, x, y, policy);
    else tma_store_2d_hint(map, buf, x, y, policy);
    bulk_commit();
  }
}

// Row-sharded grad_W: the warp's 32 x 32 chunk (times alpha) goes to the
// ranks that own its rows. The chunk is staged in shared memory in the same
// swizzled layout as for a TMA store and read back so that each warp store
// instruction writes four full 128-byte row segments; the destination is
// this rank's partial slot in the owner's buffer (plain stores, over NVLink
// for other ranks). beta == 1 accumulates into the slot (backward groups).
// Requires N and the slot leading dimension to be multiples of 4.
__device__ __forceinline__ void stage_and_scatter(uint8_t* buf, int lane, const uint32_t (&r)[32], float alpha,
                                                  const KParams& p, int col0, int row0) {
  const EpiArgs& e = p.e;
  __syncwarp();  // every lane has finished reading the previous chunk
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float4 q = make_float4(alpha * __uint_as_float(r[4 * c]), alpha * __uint_as_float(r[4 * c + 1]),
                                 alpha * __uint_as_float(r[4 * c + 2]), alpha * __uint_as_float(r[4 * c + 3]));
    *reinterpret_cast<float4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) = q;
  }
  __syncwarp();
  const int sub = lane >> 3;  // row within a group of four
  const int c = lane & 7;     // 16-byte column piece
  const int col = col0 + c * 4;
  // owner of the chunk's first row; with slices of at least 32 rows the 32
  // rows of the chunk belong to it or to the next owner (one division per
  // chunk instead of one per row)
  const long long o0 = row0 / e.slot_slice;
  const long long next0 = (o0 + 1) * e.slot_slice;
  const bool wide_slice = e.slot_slice >= 32;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int rr = it * 4 + sub;
    const long long g = static_cast<long long>(row0) + rr;
    if (g < p.M && col < p.N) {
      float4 v = *reinterpret_cast<const float4*>(buf + rr * 128 + ((c ^ (rr & 7)) << 4));
      const long long o = g < next0 ? o0 : (wide_slice ? o0 + 1 : g / e.slot_slice);
      float* dst = e.slot[o] + (static_cast<long long>(e.slot_rank) * e.slot_slice + (g - o * e.slot_slice)) * e.slot_ld +
                   col;
      if (e.beta != 0.0f) {
        const float4 old = *reinterpret_cast<const float4*>(dst);
        v.x += e.beta * old.x;
        v.y += e.beta * old.y;
        v.z += e.beta * old.z;
        v.w += e.beta * old.w;
      }
      *reinterpret_cast<float4*>(dst) = v;
    }
  }
}

// ------------------------------------------------------------------ kernel

template <int CG, bool A_MN, bool B_MN, int EPI, bool WIDE>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap mapA0, const __grid_constant__ CUtensorMap mapA1,
                const __grid_constant__ CUtensorMap mapB0, const __grid_constant__ CUtensorMap mapB1,
                const __grid_constant__ CUtensorMap mapC, const __grid_constant__ KParams p) {
  using T = TileCfg<CG, WIDE>;
  static_assert(!WIDE || EPI == static_cast<int>(Epi::Store), "wide tiles take the store epilogue");
  constexpr bool PAIR = CG == 2;
  extern __shared__ uint8_t smem_raw[];
  // Same static layout in both CTAs of a pair: the MMA reads the peer's
  // operands at the leader's offsets.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + T::STAGES * T::A_STAGE;
  uint8_t* sOut = smem + T::STAGES * T::STAGE;  // 1024-byte aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(sOut + OUT_BYTES);
  uint64_t* empty = full + T::STAGES;
  uint64_t* tfull = empty + T::STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int unit = PAIR ? static_cast<int>(cluster_id_x()) : static_cast<int>(blockIdx.x);
  const int nunits = PAIR ? static_cast<int>(num_clusters_x()) : static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], NUM_EPI_WARPS * CG);  // both CTAs' epilogues release the leader's MMA
    }
    mbar_init(drain, 1);
    fence_mbarrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&mapA0);
    tma_prefetch_desc(&mapB0);
    if (p.nseg > 1) {
      tma_prefetch_desc(&mapA1);
      tma_prefetch_desc(&mapB1);
    }
  }
  if (warp == 2) {
    tmem_alloc_cg<CG>(tmem_slot, TMEM_COLS);
    tmem_relinquish_cg<CG>();
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // peer barriers initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------- producer
    // Both CTAs of a pair load their own A rows and B half; the bytes of both
    // complete on the leader's full barrier, which the leader arms.
    const uint64_t pol_a = l2_policy(p.pol_a);
    const uint64_t pol_b = l2_policy(p.pol_b);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int w = unit; w < p.num_items && ok; w += nunits) {
      int mb, nb, kb0, kb1;
      const int tile = work_item(p, w, kb0, kb1);
      tile_coords(p, tile, mb, nb);
      const int a_row = mb * T::TILE_M + static_cast<int>(rank) * 128;
      // this CTA's B rows of MMA q start at b_row + q * BN
      const int b_row = nb * T::TILE_N + static_cast<int>(rank) * T::B_PART;
      for (int seg = 0; seg < p.nseg && ok; ++seg) {
        const CUtensorMap* ma = seg == 0 ? &mapA0 : &mapA1;
        const CUtensorMap* mbm = seg == 0 ? &mapB0 : &mapB1;
        const int k_end = kb1 < 0 ? p.seg_kblocks[seg] : kb1;
        for (int kb = kb1 < 0 ? 0 : kb0; kb < k_end; ++kb) {
          if (!mbar_wait<PAIR>(&empty[stage], phase ^ 1, p.status, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (lane == 0) {
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], T::STAGE * CG);
            const uint32_t bar = PAIR ? mapa_shared(smem_u32(&full[stage]), 0) : smem_u32(&full[stage]);
            uint8_t* a_dst = sA + stage * T::A_STAGE;
            uint8_t* b_dst = sB + stage * T::B_STAGE;
            if (!A_MN) {
              tma_load_2d_hint<CG>(a_dst, ma, bar, kb * BK, a_row, pol_a);
            } else {
#pragma unroll
              for (int i = 0; i < 128 / 64; ++i)
                tma_load_2d_hint<CG>(a_dst + i * (BK * 128), ma, bar, a_row + i * 64, kb * BK, pol_a);
            }
#pragma unroll
            for (int q = 0; q < T::NW; ++q) {
              if (!B_MN) {
                tma_load_2d_hint<CG>(b_dst + q * T::B_PART_BYTES, mbm, bar, kb * BK, b_row + q * BN, pol_b);
              } else {
#pragma unroll
                for (int i = 0; i < T::B_PART / 64; ++i)
                  tma_load_2d_hint<CG>(b_dst + q * T::B_PART_BYTES + i * (BK * 128), mbm, bar,
                                       b_row + q * BN + i * 64, kb * BK, pol_b);
              }
            }
          }
          __syncwarp();
          if (++stage == T::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1 && rank == 0) {
    // --------------------------------------------------------------- MMA
    constexpr uint32_t idesc = make_idesc_bf16_f32(T::TILE_M, BN, A_MN, B_MN);
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int w = unit; w < p.num_items && ok; w += nunits) {
      int kb0, kb1;
      work_item(p, w, kb0, kb1);
      if (!mbar_wait<PAIR>(&tempty[acc], acc_phase ^ 1, p.status, DEV_TIMEOUT_MMA)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
      bool first = true;
      for (int seg = 0; seg < p.nseg && ok; ++seg) {
        const int k_end = kb1 < 0 ? p.seg_kblocks[seg] : kb1;
        for (int kb = kb1 < 0 ? 0 : kb0; kb < k_end; ++kb) {
          if (!mbar_wait<PAIR>(&full[stage], phase, p.status, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_base = smem_u32(sA + stage * T::A_STAGE);
            const uint32_t b_base = smem_u32(sB + stage * T::B_STAGE);
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              uint64_t ad;
              if (!A_MN) ad = make_smem_desc_sw128(a_base + k * 32, 16, 1024);
              else ad = make_smem_desc_sw128(a_base + k * 2048, BK * 128, 1024);
#pragma unroll
              for (int q = 0; q < T::NW; ++q) {
                const uint32_t bq = b_base + q * T::B_PART_BYTES;
                uint64_t bd;
                if (!B_MN) bd = make_smem_desc_sw128(bq + k * 32, 16, 1024);
                else bd = make_smem_desc_sw128(bq + k * 2048, BK * 128, 1024);
                umma_bf16_cg<CG>(d_tmem + q * BN, ad, bd, idesc, (first && k == 0) ? 0u : 1u);
              }
            }
            // frees this stage in both CTAs once the MMAs have read it
            if constexpr (PAIR) umma_commit_pair(&empty[stage], 0x3);
            else umma_commit(&empty[stage]);
          }
          __syncwarp();
          first = false;
          if (++stage == T::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) break;
      if (lane == 0) {
        if constexpr (PAIR) umma_commit_pair(&tfull[acc], 0x3);
        else umma_commit(&tfull[acc]);
      }
      __syncwarp();
      if (++acc == T::NACC) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    // Drain: every MMA this thread issued has completed before teardown.
    if (lane == 0) umma_commit_cg<CG>(drain);
    __syncwarp();
    mbar_wait<PAIR>(drain, 0, p.status, DEV_TIMEOUT_DRAIN);
  } else if (warp >= EPI_WARP0) {
    // ---------------------------------------------------------- epilogue
    const int ew = warp - EPI_WARP0;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = ew >> 2;   // which 128-column half of the tile
    const int row_in_tile = static_cast<int>(rank) * 128 + quad * 32 + lane;
    const uint64_t pol_c = l2_policy(p.pol_c);
    const uint32_t tempty_leader0 = PAIR ? mapa_shared(smem_u32(&tempty[0]), 0) : 0u;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int w = unit; w < p.num_items; w += nunits) {
      int mb, nb, kb0, kb1;
      const int tile = work_item(p, w, kb0, kb1);
      // a K half of a split tile adds its partial sum into the zeroed output
      const bool split = w >= p.full_tiles && p.nsplit > 1;
      tile_coords(p, tile, mb, nb);
      if (!mbar_wait<PAIR>(&tfull[acc], acc_phase, p.status, DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const long long grow = static_cast<long long>(mb) * T::TILE_M + row_in_tile;
      const bool row_ok = grow < p.M;
      // this warp's half of the tile's columns: TMEM column j holds tile column j
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * BN + half * (T::TILE_N / 2));
      const int colh = nb * T::TILE_N + half * (T::TILE_N / 2);
      const int row0 = mb * T::TILE_M + static_cast<int>(rank) * 128 + quad * 32;
      uint8_t* buf = sOut + ew * OUT_STAGE_BYTES;
      // Releases the accumulator to the (leader's) MMA warp as soon as its
      // last TMEM load has completed (the remaining work uses registers only).
      auto release_tmem = [&]() {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if constexpr (PAIR) mbar_arrive_cluster(tempty_leader0 + static_cast<uint32_t>(acc * 8));
          else mbar_arrive(&tempty[acc]);
        }
      };
      if constexpr (EPI == static_cast<int>(Epi::Store)) {
        const float alpha = p.e.alpha_ptr ? *p.e.alpha_ptr : p.e.alpha;
        auto store = [&](int c, const uint32_t(&r)[32]) {
          const int col0 = colh + c * 32;
          if (col0 >= p.N) return;
          if (p.tma_store) {
            if (row0 < p.M) stage_and_store(buf, lane, r, alpha, &mapC, col0, row0, p.tma_reduce != 0 || split, pol_c);
          } else if (p.e.scatter) {
            if (row0 < p.M) stage_and_scatter(buf, lane, r, alpha, p, col0, row0);
          } else if (row_ok) {
            epi_store_chunk(p, grow, col0, min(32, p.N - col0), r, alpha);
          }
        };
        // the TMEM load of chunk c+1 is in flight while chunk c is stored
        constexpr int NCH = T::TILE_N / 2 / 32;
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(t_row, ra);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < NCH; c += 2) {
          tmem_ld_32x32b_x32(t_row + (c + 1) * 32, rb);
          store(c, ra);
          tmem_ld_wait();
          if (c + 2 < NCH) tmem_ld_32x32b_x32(t_row + (c + 2) * 32, ra);
          else release_tmem();
          store(c + 1, rb);
          if (c + 2 < NCH) tmem_ld_wait();
        }
      } else {
        constexpr bool OWN_DT = (EPI & 1) != 0;
        constexpr bool F16 = (EPI & 2) != 0;  // Fast profile: fp16 logits, exp2 split over SFU and FMA
        OwnStats os{-INFINITY, 0.f, 0.f, 0.f};
        const EpiArgs& e = p.e;
        auto chunk = [&](int c, const uint32_t(&r)[32]) {
          const int col0 = colh + c * 32;
          if constexpr (F16) {
            if (col0 < p.N) logits_chunk_any<OWN_DT, true>(e, grow, row_ok, col0, p.N, r, os);
            // this row's 32 values as fp16 into the staging row of a 64-column
            // pair (128 bytes, 128-byte swizzle: 16-byte piece (c & 1) * 4 + k);
            // the pair goes out in one TMA store, clipped at the tensor bounds
            if ((c & 1) == 0) {
              if (lane == 0) bulk_wait_read_all();
              __syncwarp();
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint4 q = make_uint4(pack_f16x2_sat(r[8 * k], r[8 * k + 1]), pack_f16x2_sat(r[8 * k + 2], r[8 * k + 3]),
                                         pack_f16x2_sat(r[8 * k + 4], r[8 * k + 5]),
                                         pack_f16x2_sat(r[8 * k + 6], r[8 * k + 7]));
              *reinterpret_cast<uint4*>(buf + lane * 128 + ((((c & 1) * 4 + k) ^ (lane & 7)) << 4)) = q;
            }
            if (c & 1) {
              fence_proxy_async_smem();
              __syncwarp();
              const int x = colh + (c - 1) * 32;
              if (lane == 0 && row0 < p.M && x < p.N) {
                tma_store_2d_hint(&mapC, buf, x, row0, pol_c);
                bulk_commit();
              }
            }
            return;
          }
          if (col0 >= p.N) return;
          logits_chunk_any<OWN_DT, false>(e, grow, row_ok, col0, p.N, r, os);
          if (p.tma_store) {
            if (row0 < p.M) stage_and_store(buf, lane, r, 1.0f, &mapC, col0, row0, false, pol_c);
          } else if (row_ok) {
            float* dst = static_cast<float*>(e.logits) + grow * e.ldl + col0;
            const int nv = min(32, p.N - col0);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < nv) dst[j] = __uint_as_float(r[j]);
          }
        };
        // the TMEM load of chunk c+1 is in flight while chunk c is processed
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32(t_row, ra);
        tmem_ld_wait();
        tmem_ld_32x32b_x32(t_row + 32, rb);
        chunk(0, ra);
        tmem_ld_wait();
        tmem_ld_32x32b_x32(t_row + 64, ra);
        chunk(1, rb);
        tmem_ld_wait();
        tmem_ld_32x32b_x32(t_row + 96, rb);
        chunk(2, ra);
        tmem_ld_wait();
        release_tmem();
        chunk(3, rb);
        if (row_ok && colh < p.N) {
          const long long ri = grow * e.n_parts + nb * 2 + half;
          reinterpret_cast<float4*>(e.rec_own)[ri] = make_float4(os.m, os.d1, os.dT, os.sx);
        }
      }
      if (++acc == T::NACC) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (p.tma_store && lane == 0) bulk_wait_all();
    // scattered stores reach the other ranks' memory before the kernel ends
    if (p.e.scatter) __threadfence_system();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  // A pair stays resident until the leader's MMAs (which read the peer's
  // shared memory and write its TMEM) have drained.
  if constexpr (PAIR) cluster_sync();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_cg<CG>(tmem_base, TMEM_COLS);
  }
}

// Returns the L2 lines of a matrix (rows x row_bytes, row stride ld_bytes) to
// normal eviction priority with applypriority; only whole 128-byte lines
// inside each row are touched.
__global__ void l2_demote_kernel(const uint8_t* base, long long rows, long long row_bytes, long long ld_bytes) {
  const long long lines = row_bytes / 128 + 1;  // upper bound per row
  const long long total = rows * lines;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / lines, l = i - r * lines;
    const uintptr_t row0 = reinterpret_cast<uintptr_t>(base) + static_cast<uintptr_t>(r * ld_bytes);
    const uintptr_t first = (row0 + 127) & ~uintptr_t(127);
    const uintptr_t line = first + static_cast<uintptr_t>(l) * 128;
    if (line + 128 <= row0 + static_cast<uintptr_t>(row_bytes))
      asm volatile("applypriority.global.L2::evict_normal [%0], 128;" ::"l"(line) : "memory");
  }
}

cudaError_t demote_operand(const MatRef& m, cudaStream_t stream) {
  const long long lines = m.rows * (m.cols * 2 / 128 + 1);
  if (lines <= 0) return cudaSuccess;
  const long long blocks = std::min<long long>((lines + 255) / 256, 4096);
  l2_demote_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(static_cast<const uint8_t*>(m.ptr), m.rows,
                                                                      m.cols * 2, m.ld * 2);
  return cudaGetLastError();
}

// ------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

// Encodes a 2-D bf16 map over a stored matrix (rows x cols, ld elements) with
// a box of box_inner (along cols) x box_outer (along rows), 128-byte swizzle.
bool encode_map(CUtensorMap* map, const MatRef& m, int box_inner, int box_outer) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(m.cols), static_cast<cuuint64_t>(m.rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(m.ld) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(m.ptr), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp32 output map: rows x cols with leading dimension ld (elements), 32 x 32
// box, 128-byte swizzle (the staging layout of the epilogue).
bool encode_out_map(CUtensorMap* map, float* ptr, long long rows, long long cols, long long ld) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool out_map_ok(const void* ptr, long long ld, int esz = 4) {
  return ptr && (reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && (ld * esz) % 16 == 0;
}

// fp16 logits map: rows x cols with leading dimension ld (elements), a box of
// 64 columns (128 bytes) x 32 rows, 128-byte swizzle (the staging layout of
// the Fast logits epilogue).
bool encode_out_map_f16(CUtensorMap* map, void* ptr, long long rows, long long cols, long long ld) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ptr, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Per-device, per-instantiation launch state: the shared-memory opt-in
// (a function attribute that must be set once per device) and, for CTA
// pairs, how many 2-CTA clusters can be resident at once.
struct LaunchCache {
  std::mutex mu;
  uint64_t attr_done = 0;
  int max_clusters[64] = {0};
};

// Host copy of tile_coords: the first M block among tiles [t0, num_tiles).
int first_m_block(const KParams& p, int t0) {
  int lo = p.m_blocks;
  for (int t = t0; t < p.num_tiles; ++t) {
    int mb;
    if (p.raster_n_fastest) {
      mb = t / p.n_blocks;
    } else {
      const int per_group = p.group_m * p.n_blocks;
      const int g = t / per_group;
      const int first_m = g * p.group_m;
      const int gm = std::min(p.group_m, p.m_blocks - first_m);
      mb = first_m + (t - g * per_group) % gm;
    }
    lo = std::min(lo, mb);
  }
  return lo;
}

template <int CG, bool A_MN, bool B_MN, int EPI, bool WIDE = false>
cudaError_t launch_t(const CUtensorMap* maps, const KParams& kp_in, int num_sms, cudaStream_t stream) {
  using T = TileCfg<CG, WIDE>;
  auto kern = gemm_kernel<CG, A_MN, B_MN, EPI, WIDE>;
  KParams kp = kp_in;
  static LaunchCache cache;
  int dev = 0;
  cudaGetDevice(&dev);
  dev &= 63;
  int units = num_sms / CG;
  {
    std::lock_guard<std::mutex> lock(cache.mu);
    if (!(cache.attr_done & (1ull << dev))) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, T::SMEM);
      if (e != cudaSuccess) return e;
      if (CG > 1) {
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(static_cast<unsigned>(units * CG), 1, 1);
        q.blockDim = dim3(NUM_THREADS, 1, 1);
        q.dynamicSmemBytes = T::SMEM;
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = CG;
        qa[0].val.clusterDim.y = 1;
        qa[0].val.clusterDim.z = 1;
        q.attrs = qa;
        q.numAttrs = 1;
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, kern, &q);
        if (e != cudaSuccess) return e;
        if (n <= 0) return cudaErrorInvalidConfiguration;
        cache.max_clusters[dev] = n;
      }
      cache.attr_done |= 1ull << dev;
    }
    if (CG > 1) units = cache.max_clusters[dev];
  }
  // leave kp.spare_sms SMs to kernels that run concurrently on another stream
  if (kp.spare_sms > 0) units = std::max(1, units - (kp.spare_sms + CG - 1) / CG);
  // Work items. When the last wave would leave at least half of the units
  // idle, its tiles are split into two K halves, reduce-added into the
  // output zeroed here: 0 + a + b is the same sum in either order, so the
  // result does not depend on which half lands first.
  kp.full_tiles = kp.num_tiles;
  kp.rem_tiles = 0;
  kp.nsplit = 1;
  kp.num_items = kp.num_tiles;
  {
    const int rem = kp.num_tiles % units;
    if (kp.allow_split && rem > 0 && units / rem >= 2 && kp.seg_kblocks[0] >= 2) {
      kp.full_tiles = kp.num_tiles - rem;
      kp.rem_tiles = rem;
      kp.nsplit = 2;
      kp.num_items = kp.full_tiles + 2 * rem;
      const long long r0 = static_cast<long long>(first_m_block(kp, kp.full_tiles)) * T::TILE_M;
      if (r0 < kp.M) {
        cudaError_t e = cudaMemset2DAsync(kp.e.out0 + r0 * kp.e.ld0, static_cast<size_t>(kp.e.ld0) * 4, 0,
                                          static_cast<size_t>(kp.N) * 4, static_cast<size_t>(kp.M - r0), stream);
        if (e != cudaSuccess) return e;
      }
    }
  }
  if (kp.num_items < units) units = kp.num_items;
  if (CG == 1) {
    kern<<<units, NUM_THREADS, T::SMEM, stream>>>(maps[0], maps[1], maps[2], maps[3], maps[4], kp);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(units * CG), 1, 1);
  cfg.blockDim = dim3(NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = T::SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], maps[4], kp);
}

template <int CG, bool A_MN, bool B_MN>
cudaError_t store_launch(bool wide, const CUtensorMap* maps, const KParams& kp, int num_sms, cudaStream_t stream) {
  if constexpr (CG == 2) {
    if (wide) return launch_t<CG, A_MN, B_MN, 0, true>(maps, kp, num_sms, stream);
  }
  return launch_t<CG, A_MN, B_MN, 0, false>(maps, kp, num_sms, stream);
}

template <int CG>
cudaError_t dispatch(const GemmDesc& d, const CUtensorMap* maps, const KParams& kp, int num_sms,
                     cudaStream_t stream, const char** why, bool wide) {
  if (d.epi == Epi::Logits) {
    if (d.a_mn_major || d.b_mn_major) {
      if (why) *why = "logits epilogue requires K-major operands";
      return cudaErrorInvalidValue;
    }
    // EPI code: 16 | own dT | 2 * fp16 logits
    if (d.args.logits_f16) {
      if (d.args.own_dT) return launch_t<CG, false, false, 19>(maps, kp, num_sms, stream);
      return launch_t<CG, false, false, 18>(maps, kp, num_sms, stream);
    }
    if (d.args.own_dT) return launch_t<CG, false, false, 17>(maps, kp, num_sms, stream);
    return launch_t<CG, false, false, 16>(maps, kp, num_sms, stream);
  }
  if (!d.a_mn_major && !d.b_mn_major) return store_launch<CG, false, false>(wide, maps, kp, num_sms, stream);
  if (!d.a_mn_major && d.b_mn_major) return store_launch<CG, false, true>(wide, maps, kp, num_sms, stream);
  if (d.a_mn_major && !d.b_mn_major) return store_launch<CG, true, false>(wide, maps, kp, num_sms, stream);
  return store_launch<CG, true, true>(wide, maps, kp, num_sms, stream);
}

// CTA pairs by default; ORDA_GEMM_CTA_PAIR=0 selects single-CTA tiles (a
// diagnostic switch for comparing the two tile shapes; both compute the same
// result).
bool use_cta_pair() {
  const char* v = std::getenv("ORDA_GEMM_CTA_PAIR");
  return !(v && v[0] == '0');
}

// Wide (256 x 512) pair tiles for large store-epilogue GEMMs: at least two
// waves of wide tiles over the SMs and at least 128 K blocks per tile, so
// that the per-tile epilogue, which the next tile's MMAs do not overlap,
// stays a few percent of the tile (measured at c4: dgrad, K = 2048 blocks,
// 4.8 % fewer SM cycles; wgrad, K = 128 blocks, 1.5 % fewer). A scattered
// epilogue (peer stores) is exposed in full, so it needs 1024 K blocks.
// ORDA_GEMM_WIDE=0 never uses them and ORDA_GEMM_WIDE=2 uses them for every
// store-epilogue GEMM with N > 256 (diagnostic switches; every choice
// computes the same sums, associated per tile as described at KParams).
bool use_wide(const GemmDesc& d, long long k_blocks, long long m_blocks, int num_sms) {
  const char* v = std::getenv("ORDA_GEMM_WIDE");
  const int mode = v ? (v[0] - '0') : 1;
  if (mode == 0 || d.epi != Epi::Store || d.N <= BN) return false;
  if (mode == 2) return true;
  const long long tiles = m_blocks * ((d.N + 2 * BN - 1) / (2 * BN));
  return tiles >= num_sms && k_blocks >= (d.args.scatter ? 1024 : 128);
}

}  // namespace

cudaError_t gemm_launch(const GemmDesc& d, int num_sms, cudaStream_t stream, const char** why) {
  if (why) *why = nullptr;
  if (!get_encode()) {
    if (why) *why = "cuTensorMapEncodeTiled entry point unavailable";
    return cudaErrorNotSupported;
  }
  const int cg = use_cta_pair() ? 2 : 1;
  const int tile_m = 128 * cg;
  const int b_rows = BN / cg;
  long long k_blocks = 0;
  for (int s = 0; s < d.nseg; ++s) k_blocks += (d.k_seg[s] + BK - 1) / BK;
  const bool wide = cg == 2 && use_wide(d, k_blocks, (d.M + tile_m - 1) / tile_m, num_sms);
  const int tile_n = wide ? 2 * BN : BN;
  KParams kp{};
  kp.M = static_cast<int>(d.M);
  kp.N = static_cast<int>(d.N);
  kp.m_blocks = static_cast<int>((d.M + tile_m - 1) / tile_m);
  kp.n_blocks = static_cast<int>((d.N + tile_n - 1) / tile_n);
  kp.num_tiles = kp.m_blocks * kp.n_blocks;
  kp.raster_n_fastest = d.raster_n_fastest ? 1 : 0;
  kp.nseg = d.nseg;
  kp.status = d.status;
  kp.spare_sms = d.spare_sms;
  kp.e = d.args;
  long long k_total = 0;
  CUtensorMap maps[5];
  for (int s = 0; s < 2; ++s) {
    const int src = s < d.nseg ? s : 0;
    kp.seg_kblocks[s] = s < d.nseg ? static_cast<int>((d.k_seg[s] + BK - 1) / BK) : 0;
    if (s < d.nseg) k_total += d.k_seg[s];
    const MatRef& a = d.a[src];
    const MatRef& b = d.b[src];
    for (const MatRef* m : {&a, &b}) {
      if ((reinterpret_cast<uintptr_t>(m->ptr) & 15) != 0 || (m->ld * 2) % 16 != 0 || m->ld < m->cols) {
        if (why) *why = "GEMM operand must be 16-byte aligned with ld*2 a multiple of 16";
        return cudaErrorInvalidValue;
      }
    }
    // boxes: K-major 64 (K) x rows-per-CTA; MN-major 64 (MN) x 64 (K)
    bool ok = d.a_mn_major ? encode_map(&maps[s], a, 64, BK) : encode_map(&maps[s], a, BK, 128);
    ok = ok && (d.b_mn_major ? encode_map(&maps[2 + s], b, 64, BK) : encode_map(&maps[2 + s], b, BK, b_rows));
    if (!ok) {
      if (why) *why = "cuTensorMapEncodeTiled failed";
      return cudaErrorInvalidValue;
    }
  }
  // L2 policies: an operand of at most 64 MB that is no larger than the
  // other one is re-read by every tile of its rows/columns: keep it
  // (evict-last). Outputs larger than 32 MB are written once: evict-first.
  constexpr long long kKeepBytes = 64ll << 20;
  const long long a_bytes = d.M * k_total * 2, b_bytes = d.N * k_total * 2, c_bytes = d.M * d.N * 4;
  kp.pol_a = (a_bytes <= kKeepBytes && a_bytes <= b_bytes) ? 2 : 0;
  kp.pol_b = (b_bytes <= kKeepBytes && b_bytes < a_bytes) ? 2 : 0;
  kp.pol_c = c_bytes > (32ll << 20) ? 1 : 0;
  // M-fastest raster in groups whose A slab is at most 32 MB: a wave of
  // tiles shares its B tiles, and B is re-read once per group.
  {
    const long long slab = static_cast<long long>(tile_m) * k_total * 2;
    long long g = slab > 0 ? (32ll << 20) / slab : kp.m_blocks;
    if (g < 1) g = 1;
    if (g > kp.m_blocks) g = kp.m_blocks;
    kp.group_m = static_cast<int>(g > 0 ? g : 1);
  }
  // output through shared-memory staging + TMA when the output allows it
  std::memset(&maps[4], 0, sizeof(CUtensorMap));
  kp.tma_store = 0;
  kp.tma_reduce = 0;
  if (d.args.scatter) {
    if (d.epi != Epi::Store || d.N % 4 != 0 || d.args.slot_ld % 4 != 0 || d.args.slot_slice <= 0 ||
        (d.M + d.args.slot_slice - 1) / d.args.slot_slice > kMaxSlotRanks) {
      if (why) *why = "scattered grad_W store needs a plain store, N and the slot ld multiples of 4, <= 8 owners";
      return cudaErrorInvalidValue;
    }
  } else if (d.epi == Epi::Logits) {
    if (d.args.logits_f16) {
      // the fp16 epilogue stores through TMA only
      if (!out_map_ok(d.args.logits, d.args.ldl, 2) ||
          !encode_out_map_f16(&maps[4], d.args.logits, d.M, d.N, d.args.ldl)) {
        if (why) *why = "fp16 logits need a 16-byte aligned buffer with ld a multiple of 8";
        return cudaErrorInvalidValue;
      }
      kp.tma_store = 1;
    } else if (out_map_ok(d.args.logits, d.args.ldl) &&
               encode_out_map(&maps[4], static_cast<float*>(d.args.logits), d.M, d.N, d.args.ldl)) {
      kp.tma_store = 1;
    }
  } else if (d.args.split_row >= d.M && (d.args.beta == 0.0f || d.args.beta == 1.0f) &&
             out_map_ok(d.args.out0, d.args.ld0) && encode_out_map(&maps[4], d.args.out0, d.M, d.N, d.args.ld0)) {
    kp.tma_store = 1;
    kp.tma_reduce = d.args.beta == 1.0f ? 1 : 0;
  }
  // Split tail tiles only for wide tiles: a split tile sums its K range as
  // two halves plus one add, so its rows are associated differently from
  // those of an unsplit tile of another call.
  kp.allow_split = wide && kp.tma_store && !kp.tma_reduce && d.nseg == 1 && !d.args.scatter;
  if (kp.num_tiles == 0) return cudaSuccess;
  cudaError_t e = cg == 2 ? dispatch<2>(d, maps, kp, num_sms, stream, why, wide)
                          : dispatch<1>(d, maps, kp, num_sms, stream, why, false);
  if (e != cudaSuccess) return e;
  int n = 1;
  if (d.demote_kept && (kp.pol_a == 2 || kp.pol_b == 2)) {
    for (int s = 0; s < d.nseg && e == cudaSuccess; ++s) {
      e = demote_operand(kp.pol_a == 2 ? d.a[s] : d.b[s], stream);
      ++n;
    }
  }
  if (d.launches) *d.launches += n;
  return e;
}

}  // namespace orda
