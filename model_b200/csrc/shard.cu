// Row-sharded value table over the GPUs of one node (one process per GPU).
//
// Slot s lives on rank s % world as local row s / world (striped, so a
// popular cluster of slots spreads over every rank).  After stage 2 of the
// search (the single-GPU routing kernel in routing-only mode), one forward
// is three kernels per rank, each fused with its transfer over NVLink:
//
//   scatter every (local row, weight) entry of this rank's tokens is stored
//           straight into its owner's inbox (peer memory), grouped per
//           (source rank, token) in (head, rank) order;
//   gather  each owner streams its local rows for every source rank's
//           tokens (16-byte loads, float32 accumulation; a persistent grid
//           whose warps take work from whichever source is ready) and stores
//           one partial row per (token, owner) straight into the token
//           owner's buffer -- d floats cross NVLink instead of the H*k/world rows;
//   reduce  the token owner adds the partials in rank order (deterministic)
//           and applies the SiLU gate for the output projection.
//
// Hand-off between ranks: the last CTA of a kernel (completion ticket) makes
// every CTA's peer stores visible (fence.acq_rel.sys) and release-stores
// the call's epoch into a flag in each peer's buffer; consumers acquire-load
// the flag before reading.  Every wait is bounded (about 2 s, global timer);
// on timeout the kernel records a code in the caller's status word and
// skips the work.  Buffers are reused across calls without a reset: a rank
// cannot overwrite a peer's inbox or partials before the peer has consumed
// them, because each rank's next scatter follows its own reduce, which waited
// for every owner's gather of the previous call.
#include <stdlib.h>

#include <algorithm>

#include "combine.cuh"
#include "shard.cuh"

namespace ml {

namespace {

__device__ __forceinline__ int* flag_ptr(const ShardK& S, int rank, int64_t off, int slot) {
  return reinterpret_cast<int*>(S.peer[rank] + off) + slot;
}

// Called by thread 0 of every CTA after the CTA's stores: the last CTA
// publishes the epoch into flag `flag_off`[S.hf][S.rank] of every rank (and,
// with `meta`, this half's token range into meta[S.hf][S.rank] first).
// `reset` (n ints, local) is zeroed by the last CTA for the next call: every
// CTA has finished with it once the ticket is complete.
__device__ void publish_when_last(const ShardK& S, int ticket_slot, int64_t flag_off, bool meta,
                                  int* reset = nullptr, int n_reset = 0) {
  fence_sys();
  int* ticket = reinterpret_cast<int*>(S.peer[S.rank] + S.off.tickets) + ticket_slot;
  if (atomicAdd(ticket, 1) != (int)gridDim.x - 1) return;
  *ticket = 0;   // every CTA has counted: ready for the next call
  for (int i = 0; i < n_reset; ++i) reset[i] = 0;
  fence_sys();
  const int slot = S.hf * MEMLAYER_MAX_SHARDS + S.rank;
  for (int o = 0; o < S.world; ++o) {
    if (meta) {
      *flag_ptr(S, o, S.off.meta, slot * 2) = (int)S.t0;
      *flag_ptr(S, o, S.off.meta, slot * 2 + 1) = (int)S.t1;
    }
    st_release_sys(flag_ptr(S, o, flag_off, slot), S.epoch);
  }
}

// ---------------------------------------------------------------------------
// scatter: after stage 2 has written this rank's slots and weights (the
// single-GPU routing kernel, routing only), one warp per token stores each
// (local row, weight) entry into its owner's inbox -- per owner, the
// token's entries in (head, rank) order -- and the per-owner counts
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) shard_scatter_kernel(const __grid_constant__ ShardK S, Dims D,
                                                            const int* __restrict__ slots,
                                                            const float* __restrict__ weights,
                                                            int* __restrict__ own_cnt, int* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int P = S.world, hk = S.hk;
  const unsigned lt = (1u << lane) - 1u;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t m = S.t0 + (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); m < S.t1; m += nw) {
    int run[MEMLAYER_MAX_SHARDS];   // entries of each owner so far (warp-uniform)
#pragma unroll
    for (int o = 0; o < MEMLAYER_MAX_SHARDS; ++o) run[o] = 0;
    for (int b0 = 0; b0 < hk; b0 += 32) {
      const int e = b0 + lane;
      int own = -1, lrow = 0, wbits = 0;
      if (e < hk) {
        const int sl = __ldcg(slots + m * hk + e);
        wbits = __float_as_int(__ldcg(weights + m * hk + e));
        if (sl >= 0 && (int64_t)sl < D.N) {
          // read (slot + N/2 + 1) % N under shuffle_reads (memory.py:179)
          const int64_t rs = D.shuffle ? ((int64_t)sl + D.N / 2 + 1) % D.N : (int64_t)sl;
          own = (int)(rs % P);
          lrow = (int)(rs / P);
        } else {
          atomicCAS(err, 0, 22);                 // only a bug upstream can cause this
        }
      }
      int pos = 0;
#pragma unroll
      for (int o = 0; o < MEMLAYER_MAX_SHARDS; ++o) {
        if (o >= P) break;
        const unsigned mk = __ballot_sync(FULL, own == o);
        if (own == o) pos = run[o] + __popc(mk & lt);
        run[o] += __popc(mk);
      }
      if (own >= 0)
        reinterpret_cast<int2*>(S.peer[own] + S.off.inbox)[((int64_t)S.rank * S.mcap + m) * hk + pos] =
            make_int2(lrow, wbits);
    }
#pragma unroll
    for (int o = 0; o < MEMLAYER_MAX_SHARDS; ++o) {
      if (o < P && lane == o) {
        reinterpret_cast<int*>(S.peer[o] + S.off.cnt)[(int64_t)S.rank * S.mcap + m] = run[o];
        own_cnt[m * P + o] = run[o];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) publish_when_last(S, S.hf * 2, S.off.flags_in, true);
}

// ---------------------------------------------------------------------------
// gather: a persistent grid; warps claim units of gather_tpu consecutive
// tokens of one source rank from per-source counters, taking this rank's
// own tokens first and then whichever source's inbox is ready, so a late
// push holds up only the warps that have nothing else left to do
// ---------------------------------------------------------------------------
// tokens per claimed unit: one with few sources (each token carries many
// rows), more with many (little work per token, fewer counter atomics)
__device__ __forceinline__ int gather_tpu(int world) { return world <= 2 ? 1 : world / 2; }
constexpr int GATHER_CTR = 16;   // int slot of the per-source unit counters in the tickets region

__device__ __forceinline__ int* gather_counters(const ShardK& S) {
  return reinterpret_cast<int*>(S.peer[S.rank] + S.off.tickets) + GATHER_CTR + S.hf * MEMLAYER_MAX_SHARDS;
}

// One token m of source src: its inbox entries' rows summed (float32), the
// partial row stored into the token owner's buffer.  Warp-collective.
template <typename VT, int VEC, int CH>
__device__ __forceinline__ void gather_token(const ShardK& S, const VT* __restrict__ values, int src, int64_t m,
                                             int lane, int* err) {
  const char* mine = S.peer[S.rank];
  const int d = S.d, groups = d / VEC;
  const int64_t grp = (int64_t)src * S.mcap + m;
  const int c = __ldcg(reinterpret_cast<const int*>(mine + S.off.cnt) + grp);
  if (c <= 0) return;
  const int2* ent = reinterpret_cast<const int2*>(mine + S.off.inbox) + grp * S.hk;
  float acc[CH][VEC];
#pragma unroll
  for (int a = 0; a < CH; ++a)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[a][v] = 0.f;
  for (int b0 = 0; b0 < c; b0 += 32) {
    const int2 e = (b0 + lane < c) ? __ldcg(ent + b0 + lane) : make_int2(0, 0);
    const int nb = min(32, c - b0);
#pragma unroll 4
    for (int j = 0; j < nb; ++j) {
      const int row = __shfl_sync(FULL, e.x, j);
      const float wr = __int_as_float(__shfl_sync(FULL, e.y, j));
      if ((unsigned)row >= (unsigned)S.rows) {   // only a bug upstream can cause this
        if (lane == 0) atomicCAS(err, 0, 22);
        continue;
      }
      const VT* base = values + (int64_t)row * d;
#pragma unroll
      for (int a = 0; a < CH; ++a) {
        const int g = a * 32 + lane;
        if (g < groups) {
          float x[VEC];
          load_group<VT, VEC>(base + g * VEC, x);
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[a][v] = fmaf(wr, x[v], acc[a][v]);
        }
      }
    }
  }
  // the partial goes straight to the token owner's buffer
  float* dst = reinterpret_cast<float*>(S.peer[src] + S.off.part) + ((int64_t)S.rank * S.mcap + m) * d;
#pragma unroll
  for (int a = 0; a < CH; ++a) {
    const int g = a * 32 + lane;
    if (g < groups) {
#pragma unroll
      for (int v = 0; v < VEC; v += 4)
        *reinterpret_cast<float4*>(dst + g * VEC + v) =
            make_float4(acc[a][v], acc[a][v + 1], acc[a][v + 2], acc[a][v + 3]);
    }
  }
}

template <typename VT, int VEC, int CH>
__global__ void __launch_bounds__(256) shard_gather_kernel(const __grid_constant__ ShardK S,
                                                           const VT* __restrict__ values, int* __restrict__ err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int P = S.world;
  const char* mine = S.peer[S.rank];
  const int* flags = reinterpret_cast<const int*>(mine + S.off.flags_in) + S.hf * MEMLAYER_MAX_SHARDS;
  int* ctr = gather_counters(S);
  // Sources seen ready by this CTA, and the warp that polls the flags: one
  // poller per CTA at a time, the other idle warps back off, so that waiting
  // warps do not flood L2 (where the peers' pushes land) with flag loads.
  __shared__ unsigned ready_s;
  __shared__ int poller_s;
  if (threadIdx.x == 0) {
    ready_s = 0u;
    poller_s = -1;
  }
  __syncthreads();
  const unsigned all = P >= 32 ? FULL : (1u << P) - 1u;
  unsigned done = 0, ready = 0;   // per source (bit srot), warp-uniform; `ready`: acquired by this warp
  // this rank's own tokens (its scatter ran earlier on this stream): a static
  // grid-stride pass, one token per warp step, every warp of the grid busy
  {
    int ok = 0, lo = 0, hi = 0;
    if (lane == 0 && ld_acquire_sys(flags + S.rank) - S.epoch >= 0) {
      const volatile int* meta = reinterpret_cast<const volatile int*>(mine + S.off.meta) +
                                 (S.hf * MEMLAYER_MAX_SHARDS + S.rank) * 2;
      ok = 1;
      lo = meta[0];
      hi = meta[1];
    }
    ok = __shfl_sync(FULL, ok, 0);
    if (ok) {
      lo = __shfl_sync(FULL, lo, 0);
      hi = __shfl_sync(FULL, hi, 0);
      __syncwarp();
      const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
      for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp; t < hi - lo; t += nw)
        gather_token<VT, VEC, CH>(S, values, S.rank, lo + t, lane, err);
      done = 1u;
      ready = 1u;
    }
  }
  // the other sources: units claimed from per-source counters, whichever
  // source's inbox is ready first
  long long t_idle = -1;          // lane 0: start of the current wait for any ready source
  unsigned backoff = 64;
  const int tpu = gather_tpu(P);
  while (done != all) {
    int pick = -1, u0 = 0, lo = 0, hi = 0;
    if (lane == 0) {
      for (int srot = 0; srot < P && pick < 0; ++srot) {
        if ((done >> srot) & 1u) continue;
        const int src = (S.rank + srot) % P;
        const int slot = S.hf * MEMLAYER_MAX_SHARDS + src;
        if (!((ready >> srot) & 1u)) {
          if (!((*(volatile unsigned*)&ready_s >> srot) & 1u)) continue;
          if (ld_acquire_sys(flags + src) - S.epoch < 0) continue;   // this warp's own acquire
          ready |= 1u << srot;
        }
        const volatile int* meta = reinterpret_cast<const volatile int*>(mine + S.off.meta) + slot * 2;
        const int mlo = meta[0], mhi = meta[1];
        const int c = atomicAdd(ctr + src, tpu);
        if (c >= mhi - mlo) {
          done |= 1u << srot;
          continue;
        }
        pick = srot;
        u0 = c;
        lo = mlo;
        hi = mhi;
      }
      if (pick >= 0) {
        t_idle = -1;
        backoff = 64;
      } else if (done != all) {           // no claimable source seen ready: poll or back off
        bool found = false;
        if (atomicCAS(&poller_s, -1, warp) == -1) {
          const unsigned rs = *(volatile unsigned*)&ready_s;
          for (int srot = 0; srot < P; ++srot) {
            if (((done | rs) >> srot) & 1u) continue;
            if (ld_acquire_sys(flags + (S.rank + srot) % P) - S.epoch >= 0) {
              atomicOr(&ready_s, 1u << srot);
              found = true;
            }
          }
          atomicExch(&poller_s, -1);
        }
        if (!found) {
          if (*(volatile int*)err != 0) {
            pick = -2;
          } else if (t_idle < 0) {
            t_idle = global_ns();
          } else if (global_ns() - t_idle > S.wait_ns) {   // bounded wait on the other ranks' pushes
            atomicCAS(err, 0, 31);
            pick = -2;
          } else {
            __nanosleep(backoff);
            backoff = backoff < 2048 ? backoff * 2 : 2048;
          }
        }
      }
    }
    pick = __shfl_sync(FULL, pick, 0);
    done = __shfl_sync(FULL, done, 0);
    ready = __shfl_sync(FULL, ready, 0);
    if (pick == -2) break;
    if (pick < 0) continue;
    u0 = __shfl_sync(FULL, u0, 0);
    lo = __shfl_sync(FULL, lo, 0);
    hi = __shfl_sync(FULL, hi, 0);
    __syncwarp();   // lane 0's acquire of the flag orders the warp's reads of the inbox
    const int src = (S.rank + pick) % P;
    const int tend = min(u0 + tpu, hi - lo);
    for (int t = u0; t < tend; ++t) gather_token<VT, VEC, CH>(S, values, src, lo + t, lane, err);
  }
  __syncthreads();
  if (threadIdx.x == 0) publish_when_last(S, S.hf * 2 + 1, S.off.flags_part, false, ctr, P);
}

// ---------------------------------------------------------------------------
// reduce: d/4 threads per token, float4 each
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) shard_reduce_kernel(const __grid_constant__ ShardK S, int64_t M,
                                                           const int* __restrict__ own_cnt,
                                                           const float* __restrict__ gate, float* __restrict__ out,
                                                           float* __restrict__ memg, float* __restrict__ memg_hi,
                                                           float* __restrict__ memg_lo, int* __restrict__ err) {
  const int P = S.world, d4 = S.d / 4;
  const char* mine = S.peer[S.rank];
  // thread 0 acquires every owner's flag; the barrier orders the CTA's reads after it
  __shared__ bool ok_s;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int o = 0; o < P && ok; ++o)
      ok = wait_epoch(reinterpret_cast<const int*>(mine + S.off.flags_part) + S.hf * MEMLAYER_MAX_SHARDS + o,
                      S.epoch, err, 32, S.wait_ns);
    ok_s = ok;
  }
  __syncthreads();
  const bool ok = ok_s;
  const int per = blockDim.x / d4;
  const int t = threadIdx.x / d4, i = threadIdx.x - t * d4;
  const int64_t m = S.t0 + (int64_t)blockIdx.x * per + t;
  if (!ok || t >= per || m >= S.t1) return;
  const float4* part = reinterpret_cast<const float4*>(mine + S.off.part);
  // all counts, then all partial loads in flight at once
  int cnt[MEMLAYER_MAX_SHARDS];
#pragma unroll
  for (int o = 0; o < MEMLAYER_MAX_SHARDS; ++o) cnt[o] = o < P ? own_cnt[m * P + o] : 0;
  float4 x[MEMLAYER_MAX_SHARDS];
#pragma unroll
  for (int o = 0; o < MEMLAYER_MAX_SHARDS; ++o)
    x[o] = cnt[o] > 0 ? __ldcg(part + ((int64_t)o * S.mcap + m) * d4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int o = 0; o < MEMLAYER_MAX_SHARDS; ++o) {   // owners in rank order: deterministic
    if (cnt[o] == 0) continue;
    acc.x += x[o].x;
    acc.y += x[o].y;
    acc.z += x[o].z;
    acc.w += x[o].w;
  }
  const int64_t at = m * d4 + i;
  if (out) reinterpret_cast<float4*>(out)[at] = acc;
  if (memg || memg_hi) {
    const float4 g = reinterpret_cast<const float4*>(gate)[at];      // model.py:119 mem * gate
    const float4 v = make_float4(acc.x * g.x, acc.y * g.y, acc.z * g.z, acc.w * g.w);
    if (memg) reinterpret_cast<float4*>(memg)[at] = v;
    if (memg_hi) {
      const float4 hi = make_float4(tc_round(v.x), tc_round(v.y), tc_round(v.z), tc_round(v.w));
      reinterpret_cast<float4*>(memg_hi)[at] = hi;
      reinterpret_cast<float4*>(memg_lo)[at] =
          make_float4(tc_round(v.x - hi.x), tc_round(v.y - hi.y), tc_round(v.z - hi.z), tc_round(v.w - hi.w));
    }
  }
}

// ---------------------------------------------------------------------------
// backward: probe rows out, dots back
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sigmoid_(float x) { return 1.0f / (1.0f + expf(-x)); }

// The last CTA writes `count` into slot S.rank of `meta_off` (when >= 0) and
// release-stores the epoch into slot S.rank of `flag_off`, in every rank's buffer.
__device__ void publish_backward(const ShardK& S, int ticket_slot, int64_t flag_off, int64_t meta_off, int count) {
  fence_sys();
  int* ticket = reinterpret_cast<int*>(S.peer[S.rank] + S.off.tickets) + ticket_slot;
  if (atomicAdd(ticket, 1) != (int)gridDim.x - 1) return;
  *ticket = 0;
  fence_sys();
  for (int o = 0; o < S.world; ++o) {
    if (meta_off >= 0) *flag_ptr(S, o, meta_off, S.rank) = count;
    st_release_sys(flag_ptr(S, o, flag_off, S.rank), S.epoch);
  }
}

// probe = dmemg * silu(zg), memg = mem * silu(zg), dzg = dmemg * mem * silu'(zg)
// (model.py:118-119), the same expressions as the single-GPU routing backward.
// `probe` may be `dmemg` itself (same element read, then written).
__global__ void __launch_bounds__(256) shard_probe_kernel(const __grid_constant__ ShardK S, int64_t M,
                                                          const float* dmemg, const float* __restrict__ zg,
                                                          const float* __restrict__ mem, float* probe,
                                                          float* __restrict__ memg, float* __restrict__ dzg) {
  float* mine = reinterpret_cast<float*>(S.peer[S.rank] + S.off.probe);
  const int64_t n = M * S.d;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float z = zg[i], sg = sigmoid_(z), gate = z * sg;
    const float dm = dmemg[i], mv = mem[i];
    const float p = dm * gate;
    probe[i] = p;
    mine[i] = p;
    memg[i] = mv * gate;
    dzg[i] = dm * mv * sg * (1.0f + z * (1.0f - sg));
  }
  __syncthreads();
  if (threadIdx.x == 0) publish_backward(S, 4, S.off.flags_probe, S.off.bmeta, (int)M);
}

// One warp per (source rank, token): the source's probe row crosses NVLink
// once, then probe . V[row] for each of the token's inbox entries from the
// forward (lanes over d, then a warp sum), stored into the source's dots.
template <typename VT, int VEC, int CH>
__global__ void __launch_bounds__(256) shard_dots_kernel(const __grid_constant__ ShardK S,
                                                         const VT* __restrict__ values, int* __restrict__ err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * 8 + warp;
  const int P = S.world, d = S.d;
  if (gw < (int64_t)P * S.mcap) {
    const int srot = (int)(gw / S.mcap);
    const int64_t m = gw - (int64_t)srot * S.mcap;
    const int src = (S.rank + srot) % P;
    const char* mine = S.peer[S.rank];
    bool ready = true;
    if (lane == 0) ready = wait_epoch(reinterpret_cast<const int*>(mine + S.off.flags_probe) + src, S.epoch, err, 35,
                                      S.wait_ns);
    ready = __shfl_sync(FULL, ready, 0);
    __syncwarp();
    if (ready) {
      const int64_t msrc = reinterpret_cast<const volatile int*>(mine + S.off.bmeta)[src];
      const int64_t grp = (int64_t)src * S.mcap + m;
      const int c = m < msrc ? reinterpret_cast<const volatile int*>(mine + S.off.cnt)[grp] : 0;
      if (c > 0) {
        const int groups = d / VEC;
        const float* pr = reinterpret_cast<const float*>(S.peer[src] + S.off.probe) + m * d;
        float p[CH][VEC];
#pragma unroll
        for (int a = 0; a < CH; ++a) {
          const int g = a * 32 + lane;
#pragma unroll
          for (int v = 0; v < VEC; v += 4) {
            const float4 x = g < groups ? __ldcg(reinterpret_cast<const float4*>(pr + g * VEC + v))
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
            p[a][v] = x.x;
            p[a][v + 1] = x.y;
            p[a][v + 2] = x.z;
            p[a][v + 3] = x.w;
          }
        }
        const int2* ent = reinterpret_cast<const int2*>(mine + S.off.inbox) + grp * S.hk;
        float* dst = reinterpret_cast<float*>(S.peer[src] + S.off.dots) + ((int64_t)S.rank * S.mcap + m) * S.hk;
        for (int b0 = 0; b0 < c; b0 += 32) {
          const int row_l = (b0 + lane < c) ? __ldcg(ent + b0 + lane).x : 0;
          const int nb = min(32, c - b0);
          float dot_l = 0.f;
          for (int j = 0; j < nb; ++j) {
            const int row = __shfl_sync(FULL, row_l, j);
            float acc = 0.f;
            if ((unsigned)row < (unsigned)S.rows) {
              const VT* base = values + (int64_t)row * d;
#pragma unroll
              for (int a = 0; a < CH; ++a) {
                const int g = a * 32 + lane;
                if (g < groups) {
                  float x[VEC];
                  load_group<VT, VEC>(base + g * VEC, x);
#pragma unroll
                  for (int v = 0; v < VEC; ++v) acc = fmaf(p[a][v], x[v], acc);
                }
              }
            } else if (lane == 0) {
              atomicCAS(err, 0, 22);                   // only a bug upstream can cause this
            }
            acc = warp_sum(acc);
            if (lane == j) dot_l = acc;
          }
          if (lane < nb) dst[b0 + lane] = dot_l;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) publish_backward(S, 5, S.off.flags_dots, -1, 0);
}

// ---------------------------------------------------------------------------
// staged exchange: the caller's collectives (NCCL all-gather / reduce-scatter)
// move the routing entries and the partial rows between the phases
// ---------------------------------------------------------------------------
// One warp per token of every rank (`tokens` = world * M): of the token's
// H*k (slot, weight) entries, those whose read slot this rank owns, summed in
// (head, rank) order -- the order of the owner's inbox in the peer-store
// gather, so both exchanges produce the same partial row bit for bit.
template <typename VT, int VEC, int CH>
__global__ void __launch_bounds__(256) staged_gather_kernel(Dims D, const int* __restrict__ slots,
                                                            const float* __restrict__ weights, int64_t stride,
                                                            int rank, int world, int64_t rows,
                                                            const VT* __restrict__ values,
                                                            float* __restrict__ partials, int* __restrict__ err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + warp;   // token t % M of rank t / M
  if (t >= (int64_t)world * D.M) return;
  const int hk = D.H * D.k, d = D.d, groups = d / VEC;
  const int64_t src = t / D.M;
  slots += src * stride + (t - src * D.M) * hk;
  weights += src * stride + (t - src * D.M) * hk;
  float acc[CH][VEC];
#pragma unroll
  for (int a = 0; a < CH; ++a)
#pragma unroll
    for (int v = 0; v < VEC; ++v) acc[a][v] = 0.f;
  for (int b0 = 0; b0 < hk; b0 += 32) {
    int64_t rs = 0;
    float w = 0.f;
    bool mine = false;
    if (b0 + lane < hk) {
      const int sl = __ldcg(slots + b0 + lane);
      w = __ldcg(weights + b0 + lane);
      if (sl >= 0 && (int64_t)sl < D.N) {
        rs = D.shuffle ? ((int64_t)sl + D.N / 2 + 1) % D.N : (int64_t)sl;   // memory.py:179
        mine = (int)(rs % world) == rank;
      } else {
        atomicCAS(err, 0, 22);                   // only a bug upstream can cause this
      }
    }
    const int64_t row_l = rs / world;
    unsigned mk = __ballot_sync(FULL, mine && row_l < rows);
    while (mk) {                                 // warp-uniform: entries in lane order
      const int j = __ffs(mk) - 1;
      mk &= mk - 1;
      const int64_t row = __shfl_sync(FULL, row_l, j);
      const float wr = __shfl_sync(FULL, w, j);
      const VT* base = values + row * d;
#pragma unroll
      for (int a = 0; a < CH; ++a) {
        const int g = a * 32 + lane;
        if (g < groups) {
          float x[VEC];
          load_group<VT, VEC>(base + g * VEC, x);
#pragma unroll
          for (int v = 0; v < VEC; ++v) acc[a][v] = fmaf(wr, x[v], acc[a][v]);
        }
      }
    }
  }
  float* dst = partials + t * d;
#pragma unroll
  for (int a = 0; a < CH; ++a) {
    const int g = a * 32 + lane;
    if (g < groups) {
#pragma unroll
      for (int v = 0; v < VEC; v += 4)
        *reinterpret_cast<float4*>(dst + g * VEC + v) =
            make_float4(acc[a][v], acc[a][v + 1], acc[a][v + 2], acc[a][v + 3]);
    }
  }
}

// mem * gate (model.py:119) from the reduce-scattered read output, as the
// float32 product or its tf32 halves for the tensor-core output GEMM.
__global__ void __launch_bounds__(256) staged_gate_kernel(const float4* __restrict__ mem,
                                                          const float4* __restrict__ gate, int64_t n4,
                                                          float4* __restrict__ memg, float4* __restrict__ memg_hi,
                                                          float4* __restrict__ memg_lo) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = __ldcg(mem + i), g = gate[i];
    const float4 v = make_float4(a.x * g.x, a.y * g.y, a.z * g.z, a.w * g.w);
    if (memg) memg[i] = v;
    if (memg_hi) {
      const float4 hi = make_float4(tc_round(v.x), tc_round(v.y), tc_round(v.z), tc_round(v.w));
      memg_hi[i] = hi;
      memg_lo[i] = make_float4(tc_round(v.x - hi.x), tc_round(v.y - hi.y), tc_round(v.z - hi.z), tc_round(v.w - hi.w));
    }
  }
}

inline int ch_for(int groups) {
  int ch = (groups + 31) / 32;
  return ch <= 1 ? 1 : ch <= 2 ? 2 : ch <= 4 ? 4 : ch <= 8 ? 8 : -1;
}

// Persistent grid of the gather: the CTAs that fit on the device at once
// (every CTA pays one system-scope fence), no more than there are units.
template <typename VT, int VEC, int CHV>
cudaError_t gather_launch(const ShardK& S, const VT* values, int* err, cudaStream_t s) {
  static int per_sm = 0;   // resident CTAs per SM of this instantiation (same on every B200)
  if (per_sm == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, shard_gather_kernel<VT, VEC, CHV>, 256, 0) != cudaSuccess)
      return cudaErrorInvalidValue;
    per_sm = n > 0 ? n : 1;
  }
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // enough warps for one own token each (the static pass), at most the resident CTAs
  const int64_t ctas = (S.span + 7) / 8;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ctas, (int64_t)sms * per_sm));
  shard_gather_kernel<VT, VEC, CHV><<<grid, 256, 0, s>>>(S, values, err);
  count_launch();
  return cudaGetLastError();
}

template <typename VT, int VEC>
cudaError_t gather_ch(const ShardK& S, const VT* values, int* err, cudaStream_t s) {
  switch (ch_for(S.d / VEC)) {
    case 1: return gather_launch<VT, VEC, 1>(S, values, err, s);
    case 2: return gather_launch<VT, VEC, 2>(S, values, err, s);
    case 4: return gather_launch<VT, VEC, 4>(S, values, err, s);
    case 8: return gather_launch<VT, VEC, 8>(S, values, err, s);
    default: return cudaErrorInvalidValue;
  }
}

template <typename VT, int VEC>
cudaError_t dots_ch(const ShardK& S, const VT* values, int* err, cudaStream_t s) {
  const int64_t warps = (int64_t)S.world * S.mcap;
  const unsigned grid = (unsigned)((warps + 7) / 8);
  switch (ch_for(S.d / VEC)) {
    case 1: shard_dots_kernel<VT, VEC, 1><<<grid, 256, 0, s>>>(S, values, err); break;
    case 2: shard_dots_kernel<VT, VEC, 2><<<grid, 256, 0, s>>>(S, values, err); break;
    case 4: shard_dots_kernel<VT, VEC, 4><<<grid, 256, 0, s>>>(S, values, err); break;
    case 8: shard_dots_kernel<VT, VEC, 8><<<grid, 256, 0, s>>>(S, values, err); break;
    default: return cudaErrorInvalidValue;
  }
  count_launch();
  return cudaGetLastError();
}

template <typename VT, int VEC>
cudaError_t staged_ch(const Dims& D, const int* slots, const float* weights, int64_t stride, int rank, int world,
                      int64_t rows, const VT* values, float* partials, int* err, cudaStream_t s) {
  const unsigned grid = (unsigned)(((int64_t)world * D.M + 7) / 8);
#define ML_SG(CHV) \
  staged_gather_kernel<VT, VEC, CHV><<<grid, 256, 0, s>>>(D, slots, weights, stride, rank, world, rows, values, \
                                                          partials, err)
  switch (ch_for(D.d / VEC)) {
    case 1: ML_SG(1); break;
    case 2: ML_SG(2); break;
    case 4: ML_SG(4); break;
    case 8: ML_SG(8); break;
    default: return cudaErrorInvalidValue;
  }
#undef ML_SG
  count_launch();
  return cudaGetLastError();
}

}  // namespace

ShardOff shard_layout(int world, int64_t mcap, int hk, int d) {
  auto up = [](int64_t x) { return (x + 255) / 256 * 256; };
  ShardOff o;
  o.flags_in = 0;
  o.flags_part = 256;
  o.meta = 512;
  o.tickets = 768;
  o.flags_probe = 1024;
  o.flags_dots = 1280;
  o.bmeta = 1536;
  o.cnt = 1792;
  o.inbox = o.cnt + up((int64_t)world * mcap * 4);
  o.part = o.inbox + up((int64_t)world * mcap * hk * 8);
  o.probe = o.part + up((int64_t)world * mcap * d * 4);
  o.dots = o.probe + up(mcap * d * 4);
  o.bytes = o.dots + up((int64_t)world * mcap * hk * 4);
  return o;
}

cudaError_t launch_shard_scatter(const Dims& D, const ShardK& S, const int* slots, const float* weights,
                                 int* own_cnt, int* err, cudaStream_t s) {
  // a persistent grid (every CTA pays one system-scope fence), at least one
  // CTA to publish an empty call
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ctas = (S.t1 - S.t0 + 7) / 8;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(ctas, (int64_t)sms * 8));
  shard_scatter_kernel<<<grid, 256, 0, s>>>(S, D, slots, weights, own_cnt, err);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_shard_gather(const Dims& D, const ShardK& S, const void* values, int* err, cudaStream_t s) {
  if (D.vdtype == MEMLAYER_F16) return gather_ch<__half, 8>(S, (const __half*)values, err, s);
  if (D.vdtype == MEMLAYER_BF16) return gather_ch<__nv_bfloat16, 8>(S, (const __nv_bfloat16*)values, err, s);
  return gather_ch<float, 4>(S, (const float*)values, err, s);
}

cudaError_t launch_shard_reduce(const Dims& D, const ShardK& S, const int* own_cnt, const float* gate, float* out,
                                float* memg, float* memg_hi, float* memg_lo, int* err, cudaStream_t s) {
  const int d4 = S.d / 4;
  const int per = 256 / d4;
  const int64_t n = S.t1 - S.t0;
  const unsigned grid = (unsigned)(n > 0 ? (n + per - 1) / per : 1);
  shard_reduce_kernel<<<grid, 256, 0, s>>>(S, D.M, own_cnt, gate, out, memg, memg_hi, memg_lo, err);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_shard_probe(const ShardK& S, int64_t M, const float* dmemg, const float* zg, const float* mem,
                               float* probe, float* memg, float* dzg, cudaStream_t s) {
  // at least one CTA, to publish an empty call
  const int64_t n = M * S.d;
  const int64_t blocks = (n + 255) / 256;
  const unsigned grid = (unsigned)(blocks < 1 ? 1 : blocks < 148 * 8 ? blocks : 148 * 8);
  shard_probe_kernel<<<grid, 256, 0, s>>>(S, M, dmemg, zg, mem, probe, memg, dzg);
  count_launch();
  return cudaGetLastError();
}

cudaError_t launch_shard_dots(const Dims& D, const ShardK& S, const void* values, int* err, cudaStream_t s) {
  if (D.vdtype == MEMLAYER_F16) return dots_ch<__half, 8>(S, (const __half*)values, err, s);
  if (D.vdtype == MEMLAYER_BF16) return dots_ch<__nv_bfloat16, 8>(S, (const __nv_bfloat16*)values, err, s);
  return dots_ch<float, 4>(S, (const float*)values, err, s);
}

cudaError_t launch_staged_gather(const Dims& D, const int* slots, const float* weights, int64_t stride, int rank,
                                 int world, int64_t rows, const void* values, float* partials, int* err,
                                 cudaStream_t s) {
  if (D.M <= 0) return cudaSuccess;
  if (D.vdtype == MEMLAYER_F16)
    return staged_ch<__half, 8>(D, slots, weights, stride, rank, world, rows, (const __half*)values, partials, err, s);
  if (D.vdtype == MEMLAYER_BF16)
    return staged_ch<__nv_bfloat16, 8>(D, slots, weights, stride, rank, world, rows, (const __nv_bfloat16*)values,
                                       partials, err, s);
  return staged_ch<float, 4>(D, slots, weights, stride, rank, world, rows, (const float*)values, partials, err, s);
}

cudaError_t launch_staged_gate(const float* mem, const float* gate, int64_t n, float* memg, float* memg_hi,
                               float* memg_lo, cudaStream_t s) {
  const int64_t n4 = n / 4;
  if (n4 <= 0) return cudaSuccess;
  const int64_t blocks = (n4 + 255) / 256;
  const unsigned grid = (unsigned)(blocks < 148 * 8 ? blocks : 148 * 8);
  staged_gate_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const float4*>(mem), reinterpret_cast<const float4*>(gate),
                                          n4, reinterpret_cast<float4*>(memg), reinterpret_cast<float4*>(memg_hi),
                                          reinterpret_cast<float4*>(memg_lo));
  count_launch();
  return cudaGetLastError();
}

}  // namespace ml
