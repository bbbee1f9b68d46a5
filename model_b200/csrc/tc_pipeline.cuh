// Warp-specialised TMA -> tcgen05 (3xTF32) pipeline shared by the score
// kernel and the projection GEMMs.
//
// Work is a list of units; unit u has an A row block (128 rows of a K-major
// [rows, K] float32 matrix given as hi / lo tf32 halves) and n_chunks B row
// blocks of BN rows (same K).  For every (unit, chunk) the MMA warp
// accumulates the 128 x BN product hi.hi + hi.lo + lo.hi over K in one of two
// 256-column TMEM buffers and signals tfull[buf]; the epilogue warps drain
// the buffer and signal tempty[buf].
#pragma once

#include "tc_common.cuh"

namespace ml {
namespace tc {

constexpr int PIPE_M = 128;       // rows per tile (UMMA M)
constexpr int PIPE_K = 32;        // float32 elements per 128-byte swizzled row
constexpr int PIPE_TMEM_COLS = 512;
constexpr int PIPE_ACC_STRIDE = 256;

struct PipeCtl {
  uint64_t full[8], empty[8], tfull[2], tempty[2], pair[4];
  uint32_t tmem_base;
  int abort;
};

struct PipeShape {
  int BN;          // B rows per chunk (MMA N)
  int stages;      // smem ring depth
  int bk;          // K elements per stage: 32 (128-byte swizzled rows) or 16 (64-byte)
  int kchunks;     // K / bk
  uint32_t a_bytes, b_bytes, stage_bytes;
};

// bk = 16 halves the stage size so that twice as many stages fit (deeper
// prefetch for operands read from L2).
__host__ __device__ inline PipeShape pipe_shape(int BN, int K, uint32_t extra_smem, int bk = PIPE_K) {
  PipeShape P;
  P.BN = BN;
  P.bk = bk;
  P.kchunks = K / bk;
  P.a_bytes = PIPE_M * bk * 4;
  P.b_bytes = BN * bk * 4;
  P.stage_bytes = 2 * P.a_bytes + 2 * P.b_bytes;
  const uint32_t limit = 227 * 1024;
  int st = (int)((limit - 2048 - extra_smem) / P.stage_bytes);
  P.stages = st > 6 ? 6 : st;
  return P;
}

// Barrier setup (one thread) and TMEM allocation (warp 1); all threads call.
__device__ __forceinline__ uint32_t pipe_init(PipeCtl* ctl, const PipeShape& P, int epi_warps) {
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < P.stages; ++s) {
      mbar_init(&ctl->full[s], 1);
      mbar_init(&ctl->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->tfull[b], 1);
      mbar_init(&ctl->tempty[b], epi_warps);
    }
    for (int q = 0; q < 4; ++q) mbar_init(&ctl->pair[q], 2);
    ctl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&ctl->tmem_base, PIPE_TMEM_COLS);
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  return ctl->tmem_base;
}

__device__ __forceinline__ void pipe_finish(PipeCtl* ctl, uint32_t tmem_base) {
  fence_before_sync();
  __syncthreads();
  if ((threadIdx.x >> 5) == 1) {
    fence_after_sync();
    tmem_dealloc(tmem_base, PIPE_TMEM_COLS);
  }
}

// Producer (one thread).  coords(u, &arow, &brow0, &nchunks).  With wrap > 0
// chunk j of a unit reads B rows from chunk j % wrap (a unit that passes
// over the same B rows several times).
template <class Coords>
__device__ __forceinline__ void pipe_produce(PipeCtl* ctl, const PipeShape& P, uint8_t* tiles, int units,
                                             const CUtensorMap* tA_hi, const CUtensorMap* tA_lo,
                                             const CUtensorMap* tB_hi, const CUtensorMap* tB_lo, Coords coords,
                                             int* err, int wrap = 0) {
  volatile int* abort = &ctl->abort;
  prefetch_tmap(tA_hi);
  prefetch_tmap(tA_lo);
  prefetch_tmap(tB_hi);
  prefetch_tmap(tB_lo);
  int s = 0;
  uint32_t ph = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    int arow, brow0, nch;
    coords(u, arow, brow0, nch);
    for (int j = 0; j < nch; ++j) {
      const int brow = brow0 + (wrap > 0 ? j % wrap : j) * P.BN;
      for (int kc = 0; kc < P.kchunks; ++kc) {
        if (!mbar_wait(&ctl->empty[s], ph ^ 1, abort, err, 11)) return;
        uint8_t* st = tiles + (size_t)s * P.stage_bytes;
        mbar_expect_tx(&ctl->full[s], P.stage_bytes);
        tma_load_2d(st, tA_hi, &ctl->full[s], kc * P.bk, arow);
        tma_load_2d(st + P.a_bytes, tA_lo, &ctl->full[s], kc * P.bk, arow);
        tma_load_2d(st + 2 * P.a_bytes, tB_hi, &ctl->full[s], kc * P.bk, brow);
        tma_load_2d(st + 2 * P.a_bytes + P.b_bytes, tB_lo, &ctl->full[s], kc * P.bk, brow);
        if (++s == P.stages) {
          s = 0;
          ph ^= 1;
        }
      }
    }
  }
}

// MMA issuer (one thread).
template <class Coords>
__device__ __forceinline__ void pipe_mma(PipeCtl* ctl, const PipeShape& P, uint8_t* tiles, int units,
                                         uint32_t tmem_base, Coords coords, int* err) {
  volatile int* abort = &ctl->abort;
  const uint32_t idesc = idesc_tf32(PIPE_M, P.BN);
  int s = 0, acc = 0;
  uint32_t ph = 0, aph = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x) {
    int arow, brow0, nch;
    coords(u, arow, brow0, nch);
    for (int j = 0; j < nch; ++j) {
      if (!mbar_wait(&ctl->tempty[acc], aph ^ 1, abort, err, 12)) return;
      fence_after_sync();
      const uint32_t d = tmem_base + (uint32_t)(acc * PIPE_ACC_STRIDE);
      for (int kc = 0; kc < P.kchunks; ++kc) {
        if (!mbar_wait(&ctl->full[s], ph, abort, err, 13)) return;
        fence_after_sync();
        const uint32_t a_hi = smem_u32(tiles + (size_t)s * P.stage_bytes);
        const uint32_t a_lo = a_hi + P.a_bytes, b_hi = a_hi + 2 * P.a_bytes, b_lo = b_hi + P.b_bytes;
        if (P.bk == PIPE_K) {
#pragma unroll
          for (int k8 = 0; k8 < PIPE_K / 8; ++k8) {
            const uint32_t off = k8 * 32;  // 8 tf32 = 32 bytes along K inside the swizzled row
            const uint64_t dah = sdesc_k_sw128(a_hi + off), dal = sdesc_k_sw128(a_lo + off);
            const uint64_t dbh = sdesc_k_sw128(b_hi + off), dbl = sdesc_k_sw128(b_lo + off);
            mma_tf32(d, dah, dbh, idesc, (kc | k8) != 0);
            mma_tf32(d, dah, dbl, idesc, 1);
            mma_tf32(d, dal, dbh, idesc, 1);
          }
        } else {
#pragma unroll
          for (int k8 = 0; k8 < 2; ++k8) {     // 16 tf32 = one 64-byte swizzled row
            const uint32_t off = k8 * 32;
            const uint64_t dah = sdesc_k_sw64(a_hi + off), dal = sdesc_k_sw64(a_lo + off);
            const uint64_t dbh = sdesc_k_sw64(b_hi + off), dbl = sdesc_k_sw64(b_lo + off);
            mma_tf32(d, dah, dbh, idesc, (kc | k8) != 0);
            mma_tf32(d, dah, dbl, idesc, 1);
            mma_tf32(d, dal, dbh, idesc, 1);
          }
        }
        mma_commit(&ctl->empty[s]);  // the stage is free once these MMAs have read it
        if (++s == P.stages) {
          s = 0;
          ph ^= 1;
        }
      }
      mma_commit(&ctl->tfull[acc]);  // accumulator complete
      acc ^= 1;
      if (acc == 0) aph ^= 1;
    }
  }
}

// Bounded rendezvous of the two epilogue warps that share a TMEM lane quarter.
__device__ __forceinline__ bool pair_sync(uint64_t* bar, uint32_t& parity, int lane, volatile int* abort, int* err) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
  const bool ok = mbar_wait(bar, parity, abort, err, 15);
  parity ^= 1;
  return __all_sync(FULL, ok);
}

}  // namespace tc
}  // namespace ml
