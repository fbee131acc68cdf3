// apx_gemv.cu — exact Q8-activation GEMV for GGUF Q8_0 / Q4_K / Q6_K on sm_100a.
//
// Contract (src/engine/chart/mod.rs:1887-1925): out[r] = round_shift_32(Σ_i w_ri·x̂_i) with
// w the Q32.32 dequantized weight and x̂_i = S_b·xq_i, i.e. `matvec_fixed(W, dequant(q))`
// (src/engine/ops/matvec.rs:149-222), bit for bit, with the same refusals.
//
// Layout in HBM.  At upload each tensor is regrouped once into units of 32 lanes.  A K-slot
// is 4 Q8_0 blocks or one Q4_K / Q6_K super-block; lane l of unit (rt, j) holds row
// rt·H + l/L, K-slot j·L + l%L, where L (1, 2 or 4) lanes share a row and H = 32/L rows
// form a row tile.  Inside a unit the 16-byte chunk c of lane l sits at (c*32 + l)*16, so
// every warp-wide 16-byte load reads 512 contiguous bytes; the per-row block headers follow
// the chunks.  The bytes are the GGUF bytes, only their positions change (format/quant.rs:
// 52-68 block layouts).  L > 1 is chosen for few, long rows (down projections), so a row's
// K-slots spread over lanes instead of over CTAs.
//
// Work.  One warp folds one unit: each lane accumulates its slot of its row exactly in a
// 128-bit integer (apx_common.cuh); the L lanes of a row combine by shuffles, the warps of a
// row tile in shared memory.  Matrices that fit one resident wave use one unit per warp
// (every load in flight at once); larger ones use a persistent kernel in which each warp
// streams a contiguous chunk of units with one unit of prefetch.
//
// Exactness.  The kernels run when every partial sum is provably inside i128 (the reference's
// call-level bound q8act_fast_bound_ok, chart/mod.rs:362-383, evaluated from the largest
// activation exponent) and the activation exponent spread fits the family's i64 super-block
// fold; otherwise the same kernel takes the checked path, one lane per row summing
// Σ w_i·x̂_i in element order with i128 overflow detection, which is matvec_fixed itself.
#include <algorithm>
#include <cstdlib>

#include "apx_common.cuh"
#include "apx_kernels.h"
#include "apx_pack.cuh"
#include "apx_unit.cuh"

namespace apx {

// K-slots per row: Q8_0 counts quads of 32-lane blocks, the k-quants super-blocks.
int units_per_row_tile(uint32_t type, size_t n_in) {
  if (type == kQ8_0) return (int)((((n_in + 31) / 32) + 3) / 4);
  return (int)((n_in + 255) / 256);
}

// ---- upload-time repack ----------------------------------------------------------------

__global__ void repack_kernel(const uint8_t *__restrict__ raw, uint8_t *__restrict__ pack,
                              uint32_t type, size_t n_out, size_t row_bytes, int units, int L,
                              int kslots, int nblk, size_t total) {
  const int H = 32 / L;
  const int unit_bytes = unit_bytes_of(type);
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const size_t unit = idx / unit_bytes;
    const int off = (int)(idx % unit_bytes);
    const size_t rt = unit / units;
    const int j = (int)(unit % units);
    int lane, within;  // lane, and byte offset inside that lane's K-slot of the GGUF row
    if (type == kQ8_0) {
      if (off < 4096) {
        lane = (off / 16) % 32;
        const int c = off / 512;  // block c/2 of the slot, half c%2
        within = (c / 2) * 34 + 2 + 16 * (c % 2) + off % 16;
      } else {
        lane = (off - 4096) / 8;
        within = ((off - 4096) % 8 / 2) * 34 + (off - 4096) % 2;
      }
    } else if (type == kQ4_K) {
      if (off < 4096) {
        lane = (off / 16) % 32;
        within = 16 + 16 * (off / 512) + off % 16;
      } else {
        lane = (off - 4096) / 16;
        within = (off - 4096) % 16;
      }
    } else {
      if (off < 6144) {
        lane = (off / 16) % 32;
        within = 16 * (off / 512) + off % 16;
      } else if (off < 6656) {
        lane = (off - 6144) / 16;
        within = 192 + (off - 6144) % 16;
      } else {
        lane = (off - 6656) / 2;
        within = 208 + (off - 6656) % 2;
      }
    }
    const size_t row = rt * H + lane / L;
    const int slot = j * L + lane % L;
    bool valid = row < n_out && slot < kslots;
    size_t src = 0;
    if (type == kQ8_0) {
      const int blk = 4 * slot + within / 34;
      valid = valid && blk < nblk;
      src = (size_t)slot * 4 * 34 + within;
    } else {
      src = (size_t)slot * (type == kQ4_K ? 144 : 210) + within;
    }
    pack[idx] = valid ? raw[row * row_bytes + src] : (uint8_t)0;
  }
}

// ---- the one-wave kernel --------------------------------------------------------------------

struct GemvArgs {
  const uint8_t *pack;
  int units;        // units per row tile
  int L;            // lanes per row
  size_t n_rt;      // row tiles (of 32/L rows)
  size_t n_out, n_in;
  const int8_t *codes;
  const uint8_t *exps;
  const ActDesc *desc;
  long long *out_q32;
  float *out_f32;
  unsigned long long *status;
  Acc128 *partials;     // [n_rt][ksplit][32] partial sums of a K-split row tile
  unsigned *counters;   // [n_rt] arrivals of a K-split row tile (self-resetting)
  int R, P, ksplit;     // row tiles per CTA, warps per row tile, CTAs per row tile along K
  int cluster;          // > 1: the ksplit CTAs of a row tile are one cluster (R = 1)
  int w_off;            // shared offset of the warps' weight slots (one unit each)
  int act_bytes;        // shared bytes of the activation staging / partial sums
  PeerRows peers;       // also store the outputs there (row-sharded gather), n = 0 otherwise
  GemvGroup grp;        // several tensors sharing the activation, n = 0 otherwise
};

// The group member holding the launch's row tile grt: its weights and its local row tile.
// Constant indices throughout, so the parameter block stays in the constant bank.
__device__ __forceinline__ void group_member(const GemvGroup &grp, size_t grt, size_t &rt,
                                             const uint8_t *&pack) {
#pragma unroll
  for (int t = 0; t < kMaxGroup; t++) {
    const size_t begin = t ? grp.rt_end[t - 1] : 0;
    if (t < grp.n && grt >= begin && grt < grp.rt_end[t]) {
      rt = grt - begin;
      pack = grp.pack[t];
    }
  }
}

struct GroupOut {
  size_t n_out;
  long long *q32;
  float *f32;
  unsigned long long *status;
};

__device__ __forceinline__ GroupOut group_outputs(const GemvGroup &grp, size_t grt) {
  GroupOut o{0, nullptr, nullptr, nullptr};
#pragma unroll
  for (int t = 0; t < kMaxGroup; t++) {
    const size_t begin = t ? grp.rt_end[t - 1] : 0;
    if (t < grp.n && grt >= begin && grt < grp.rt_end[t])
      o = GroupOut{grp.n_out[t], grp.out_q32[t], grp.out_f32[t], grp.status[t]};
  }
  return o;
}

// kSmemW: the unit goes into a shared-memory slot by cp.async instead of into registers (see
// the two kernels after the body).
template <uint32_t T, bool kSmemW>
__device__ __forceinline__ void gemv_body(const GemvArgs &g) {
  extern __shared__ __align__(16) unsigned char smem[];
  using F = Fam<T>;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int ks = (int)(blockIdx.x % g.ksplit);
  // this CTA's row tiles [rt0, rt1): an even share of the n_rt over the grid's rows of CTAs,
  // at most R
  // (one-wave plans keep n_rt·grid below 2^32)
  const unsigned cta_row = blockIdx.x / g.ksplit, grid_rows = gridDim.x / g.ksplit;
  const size_t rt0 = cta_row * (unsigned)g.n_rt / grid_rows;
  const size_t rt1 = (cta_row + 1) * (unsigned)g.n_rt / grid_rows;
  const int nr = (int)(rt1 - rt0);
  const int k0 = (int)((long long)g.units * ks / g.ksplit);
  const int k1 = (int)((long long)g.units * (ks + 1) / g.ksplit);
  const int r = warp / g.P, p = warp % g.P;
  const bool active = r < nr;
  // this warp's tensor: the launch's own, or the group member holding row tile rt0 + r (its
  // outputs are selected again at the finish, so they hold no registers through the fold)
  size_t rt = rt0 + r;
  const uint8_t *pack = g.pack;
  if (g.grp.n) group_member(g.grp, rt0 + r, rt, pack);
  const uint8_t *base = pack + rt * (size_t)g.units * F::unit_bytes;
  const int L = g.L, H = 32 / L, slot = lane % L;
  const int nch = L * F::span / 16;  // chunks staged per unit: 8, 16, 32 or 64
  // a cluster's CTAs store into CTA 0's shared memory at the end: each arrives here, and
  // waits there for the others, so that none is written before it has started
  if (g.cluster > 1) cluster_arrive_relaxed();

  pdl_launch_dependents();
  // weights first: they depend on nothing the previous kernel writes, and the plan gives every
  // warp at most one unit (k1 - k0 <= P).  Into registers, or copied into this warp's
  // shared-memory slot without passing through registers.
  uint8_t *wslot = smem + g.w_off + (size_t)warp * F::unit_bytes;
  UnitRegs<T> cur;
  const bool first = active && k0 + p < k1;
  if (first) {
    const uint8_t *src = base + (size_t)(k0 + p) * F::unit_bytes;
    if (kSmemW) {
      for (int i = lane; i < F::unit_bytes / 16; i += 32)
        cp_async16(wslot + (size_t)i * 16, src + (size_t)i * 16);
    } else {
      load_unit(cur, src, lane);
    }
  }
  if (kSmemW) cp_async_commit();
  pdl_wait();

  // the descriptor and this warp's activation chunks in one round trip
  const ActDesc desc = *g.desc;
  Chunk ch0 = {make_uint4(0, 0, 0, 0), APX_EXP_ZERO}, ch1 = ch0;
  if (first) {
    if (lane < nch) ch0 = load_chunk(g.codes, g.exps, g.n_in, chunk_first<T>(k0 + p, L, lane));
    if (lane + 32 < nch)
      ch1 = load_chunk(g.codes, g.exps, g.n_in, chunk_first<T>(k0 + p, L, lane + 32));
  }
  if (desc.status != APX_OK) {  // the activation itself is refused (chart/mod.rs:1904-1907)
    if (kSmemW) cp_async_wait_all();  // no copy lands after the CTA exits
    if (blockIdx.x == 0 && threadIdx.x == 0) {
      if (!g.grp.n) atomicMin(g.status, pack_status(0, (unsigned)desc.status, 0));
#pragma unroll
      for (int t = 0; t < kMaxGroup; t++)
        if (t < g.grp.n) atomicMin(g.grp.status[t], pack_status(0, (unsigned)desc.status, 0));
    }
    return;
  }
  // the fast fold within the family's spread limit, the wide one beyond it while the call
  // bound holds, the checked rows otherwise
  const bool wide = !fast_path<T>(desc, g.n_in);
  if (wide && !wide_path<T>(desc, g.n_in)) {
    if (kSmemW) cp_async_wait_all();
    if (ks == 0 && p == 0 && active && slot == 0) {
      GroupOut go{g.n_out, g.out_q32, g.out_f32, g.status};
      if (g.grp.n) go = group_outputs(g.grp, rt0 + r);
      const RowOut o = checked_row<T>(PackGeo{pack, g.units, L}, rt * H + lane / L, go.n_out,
                                      g.n_in, g.codes, g.exps, go.q32, go.f32, go.status);
      if (o.ok) store_peers(g.peers, rt * H + lane / L, o.v);
    }
    return;
  }

  // -- fold this warp's unit ------------------------------------------------------------------
  WarpAct<T> *w = reinterpret_cast<WarpAct<T> *>(smem) + warp;
  Acc128 acc;
  acc_zero(acc);
  if (first) {
    store_chunk<T>(*w, ch0, lane, lane < nch, desc.emin, wide);
    if (nch > 32) store_chunk<T>(*w, ch1, lane + 32, lane + 32 < nch, desc.emin, wide);
    if (kSmemW) {
      cp_async_wait_all();
      __syncwarp();  // every lane's staging and weight copies before any lane's fold
      fold_unit_smem<T>(acc, wslot, lane, w->codes + slot * slot_ints<T>(),
                        w->e + slot * (F::span / 32), w->xs + slot * F::nxs, desc.emin, wide);
    } else {
      __syncwarp();
      if (wide)
        fold_unit_wide(acc, cur, w->codes + slot * slot_ints<T>(), w->e + slot * (F::span / 32),
                       w->xs + slot * F::nxs, desc.emin);
      else
        fold_unit(acc, cur, w->codes + slot * slot_ints<T>(), w->e + slot * (F::span / 32),
                  w->xs + slot * F::nxs, desc.emin);
    }
  } else if (kSmemW) {
    cp_async_wait_all();
  }
  // the L lanes of a row combine
  for (int o = 1; o < L; o <<= 1) {
    const unsigned long long lo = __shfl_xor_sync(0xFFFFFFFFu, acc.lo, o);
    const unsigned long long hi = __shfl_xor_sync(0xFFFFFFFFu, acc.hi, o);
    acc_add(acc, lo, hi);
  }

  // -- reduce: warps of a row tile in shared memory, CTAs of a row tile through scratch ----
  __syncthreads();  // the staging region is reused for the partial sums
  Acc128 *part = reinterpret_cast<Acc128 *>(smem);  // [R*P][32]
  part[warp * 32 + lane] = acc;
  __syncthreads();
  Acc128 s;
  acc_zero(s);
  if (p == 0 && r < nr) {
    s = part[(r * g.P) * 32 + lane];
    for (int q = 1; q < g.P; q++) acc_add(s, part[(r * g.P + q) * 32 + lane]);
  }
  bool finalize = ks == 0;
  if (g.cluster > 1) {
    // the row tile's CTAs are one cluster (R = 1): each stores its partial into CTA 0's shared
    // memory, and CTA 0 sums them once the cluster barrier has seen every store
    Acc128 *slots = reinterpret_cast<Acc128 *>(smem + g.act_bytes);  // [ksplit][32]
    cluster_wait_acquire();  // every CTA of the cluster has started
    if (p == 0 && active) st_cluster_acc(cluster_map(slots + ks * 32 + lane, 0), s.lo, s.hi);
    cluster_arrive_release();
    if (ks != 0) return;
    cluster_wait_acquire();
    if (p == 0 && active) {
      acc_zero(s);
      for (int q = 0; q < g.ksplit; q++) acc_add(s, slots[q * 32 + lane]);
    }
  } else if (g.ksplit > 1) {
    // last-arriving CTA of the row tile sums the others' partials (threadfence reduction)
    unsigned *ticket = reinterpret_cast<unsigned *>(part + g.R * g.P * 32);
    if (p == 0 && active) {
      Acc128 *dst = g.partials + (rt * g.ksplit + ks) * 32 + lane;
      dst->lo = s.lo;
      dst->hi = s.hi;
      __threadfence();
    }
    __syncthreads();
    if (threadIdx.x < (unsigned)g.R)
      ticket[threadIdx.x] = (int)threadIdx.x < nr
                                ? atomicAdd(g.counters + rt0 + threadIdx.x, 1u)
                                : 0u;
    __syncthreads();
    finalize = active && ticket[r] == (unsigned)(g.ksplit - 1);
    if (finalize && p == 0) {
      __threadfence();
      acc_zero(s);
      for (int q = 0; q < g.ksplit; q++) {
        const Acc128 *src = g.partials + (rt * g.ksplit + q) * 32 + lane;
        acc_add(s, __ldcg(&src->lo), __ldcg(&src->hi));
      }
      if (lane == 0) g.counters[rt] = 0u;  // ready for the next call
    }
  }
  if (finalize && p == 0 && active && slot == 0) {
    GroupOut go{g.n_out, g.out_q32, g.out_f32, g.status};
    if (g.grp.n) go = group_outputs(g.grp, rt0 + r);
    finish_row(s, rt * H + lane / L, go.n_out, go.q32, go.f32, go.status, g.peers);
  }
}

// Weights in registers (80 a thread): one CTA of a projection and one of the next fill an SM.
template <uint32_t T>
__global__ void __launch_bounds__(384, 2) gemv_kernel(GemvArgs g) {
  gemv_body<T, false>(g);
}
// Weights in shared memory (64 registers a thread): for a plan whose CTAs would not all be
// resident at 80 registers (a second wave of a few CTAs costs a whole dependency chain).
template <uint32_t T>
__global__ void __maxnreg__(64) gemv_kernel_smem(GemvArgs g) {
  gemv_body<T, true>(g);
}

// ---- streaming kernel for matrices larger than one resident wave ---------------------------
//
// Persistent (L = 1): V = gridDim.x × warps-per-CTA warps, warp v streams the contiguous unit
// chunk [v·C, (v+1)·C) of the (row tile, K unit) order, C = ceil(T/V), folding one unit while
// the next is in flight.  The CTA stages the whole activation once.  A row tile covered by
// one warp is finished by it; a row tile split between warps is finished by whichever of them
// arrives last (partial sums in the tensor's scratch, an arrival counter that resets itself).

struct StreamArgs {
  const uint8_t *pack;
  int units;          // U, units per row tile
  size_t n_rt, n_out, n_in;
  const int8_t *codes;
  const uint8_t *exps;
  const ActDesc *desc;
  long long *out_q32;
  float *out_f32;
  unsigned long long *status;
  Acc128 *partials;   // [n_rt][kmax][32]
  unsigned *counters; // [n_rt]
  long long chunk;    // C
  int kmax;           // most warps that can share a row tile
  PeerRows peers;     // also store the outputs there (row-sharded gather), n = 0 otherwise
};

// Q6_K holds 53 registers of weights per unit (two with the prefetch): one CTA of 12 warps per
// SM gives it the registers; the other families run two CTAs of 8 warps.
template <uint32_t T>
__host__ __device__ constexpr int stream_threads() { return T == kQ6_K ? 384 : 256; }

template <uint32_t T>
__global__ void __launch_bounds__(stream_threads<T>(), T == kQ6_K ? 1 : 2)
    gemv_stream_kernel(StreamArgs g) {
  extern __shared__ __align__(16) unsigned char smem[];
  using F = Fam<T>;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  const long long U = g.units, Ttot = (long long)g.n_rt * U;
  const long long v = (long long)blockIdx.x * nw + warp;
  const long long x0 = v * g.chunk, x1 = min(Ttot, x0 + g.chunk);

  pdl_launch_dependents();
  UnitRegs<T> cur;
  if (x0 < x1) load_unit(cur, g.pack + (size_t)x0 * F::unit_bytes, lane);
  pdl_wait();

  const ActDesc desc = *g.desc;
  if (desc.status != APX_OK) {
    if (blockIdx.x == 0 && threadIdx.x == 0)
      atomicMin(g.status, pack_status(0, (unsigned)desc.status, 0));
    return;
  }
  const bool wide = !fast_path<T>(desc, g.n_in);  // as in gemv_kernel
  if (wide && !wide_path<T>(desc, g.n_in)) {
    // the warp holding a row tile's first unit runs that tile's checked rows
    for (long long x = x0; x < x1; x++) {
      if (x % U != 0) continue;
      const RowOut o = checked_row<T>(PackGeo{g.pack, g.units, 1}, (size_t)(x / U) * 32 + lane,
                                      g.n_out, g.n_in, g.codes, g.exps, g.out_q32, g.out_f32,
                                      g.status);
      if (o.ok) store_peers(g.peers, (size_t)(x / U) * 32 + lane, o.v);
    }
    return;
  }

  // -- the whole activation, staged once per CTA ---------------------------------------
  const int nel = (int)U * F::span;
  int *s_codes = reinterpret_cast<int *>(smem);
  int *s_e = s_codes + nel / 4;
  long long *s_xs = reinterpret_cast<long long *>(s_e + ((nel / 32 + 3) & ~3));
  const int n16 = nel / 16;
  for (int base = 0; base < n16; base += blockDim.x) {  // whole warps: the shuffle below
    const int j16 = base + threadIdx.x;
    const bool in = j16 < n16;
    const Chunk ch = in ? load_chunk(g.codes, g.exps, g.n_in, 16 * (size_t)j16)
                        : Chunk{make_uint4(0, 0, 0, 0), APX_EXP_ZERO};
    const bool zero = ch.e == APX_EXP_ZERO;
    const uint4 val = zero ? make_uint4(0, 0, 0, 0) : ch.v;
    const int er = zero ? 0 : (int)ch.e - desc.emin;
    int s16 = dp4a_ss((int)val.x, 0x01010101, 0);
    s16 = dp4a_ss((int)val.y, 0x01010101, s16);
    s16 = dp4a_ss((int)val.z, 0x01010101, s16);
    s16 = dp4a_ss((int)val.w, 0x01010101, s16);
    const int s32 = s16 + __shfl_xor_sync(0xFFFFFFFFu, s16, 1);
    if (!in) continue;
    reinterpret_cast<uint4 *>(s_codes)[j16] = val;
    if (T == kQ6_K) s_xs[j16] = wide ? (long long)s16 : (long long)s16 << er;
    if ((j16 & 1) == 0) {
      s_e[j16 / 2] = T == kQ8_0 ? (zero ? -1 : (int)ch.e) : er;
      if (T == kQ4_K) s_xs[j16 / 2] = s32;
    }
  }
  __syncthreads();

  // -- stream the chunk ---------------------------------------------------------------------
  Acc128 acc;
  acc_zero(acc);
  // the unit's row tile and K position advance with it (no division per unit)
  long long rt = x0 / U;
  int u = (int)(x0 - rt * U);
  const uint8_t *next_unit = g.pack + (size_t)(x0 + 1) * F::unit_bytes;
  for (long long x = x0; x < x1; x++, next_unit += F::unit_bytes) {
    UnitRegs<T> nxt;
    const bool more = x + 1 < x1;
    if (more) load_unit(nxt, next_unit, lane);
    if (wide)
      fold_unit_wide(acc, cur, s_codes + u * (F::span / 4), s_e + u * (F::span / 32),
                     s_xs + u * F::nxs, desc.emin);
    else
      fold_unit(acc, cur, s_codes + u * (F::span / 4), s_e + u * (F::span / 32),
                s_xs + u * F::nxs, desc.emin);
    if (u == U - 1 || !more) {
      // flush this warp's share of row tile rt
      const long long first_v = (rt * U) / g.chunk;
      const long long last_v = (rt * U + U - 1) / g.chunk;
      const size_t row = (size_t)rt * 32 + lane;
      if (first_v == last_v) {
        finish_row(acc, row, g.n_out, g.out_q32, g.out_f32, g.status, g.peers);
      } else {
        const int k = (int)(v - first_v), count = (int)(last_v - first_v + 1);
        Acc128 *slot = g.partials + ((size_t)rt * g.kmax + k) * 32 + lane;
        slot->lo = acc.lo;
        slot->hi = acc.hi;
        __syncwarp();  // the lanes' stores, then lane 0's release fence and arrival
        fence_acq_rel_gpu();
        unsigned ticket = 0;
        if (lane == 0) ticket = atomicAdd(g.counters + rt, 1u);
        ticket = __shfl_sync(0xFFFFFFFFu, ticket, 0);
        if (ticket == (unsigned)(count - 1)) {
          fence_acq_rel_gpu();  // lane 0's acquire, then the lanes' loads
          __syncwarp();
          Acc128 s;
          acc_zero(s);
          for (int q = 0; q < count; q++) {
            const Acc128 *src = g.partials + ((size_t)rt * g.kmax + q) * 32 + lane;
            acc_add(s, __ldcg(&src->lo), __ldcg(&src->hi));
          }
          finish_row(s, row, g.n_out, g.out_q32, g.out_f32, g.status, g.peers);
          if (lane == 0) g.counters[rt] = 0u;
        }
      }
      acc_zero(acc);
    }
    if (more) cur = nxt;
    if (++u == U) {
      u = 0;
      rt++;
    }
  }
}

// ---- exact int32 group dots from the repacked layout (parity hook) -------------------------

__global__ void block_dots_kernel(uint32_t type, PackGeo geo, size_t n_out, size_t per_row,
                                  const int8_t *codes, int32_t *dots) {
  const size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (idx >= n_out * per_row) return;
  const size_t row = idx / per_row, g = idx % per_row;
  int lane, dot = 0;
  if (type == kQ8_0) {
    const uint8_t *ub = slot_unit(geo, type, row, g / 4, lane);
    const int bi = (int)(g % 4);
    for (int qi = 0; qi < 32; qi++) {
      const int c = 2 * bi + qi / 16;
      dot += (int)(signed char)ub[(c * 32 + lane) * 16 + qi % 16] * codes[g * 32 + qi];
    }
  } else if (type == kQ4_K) {
    const size_t s = g / 8;
    const int grp = (int)(g % 8);
    const uint8_t *ub = slot_unit(geo, type, row, s, lane);
    for (int l = 0; l < 32; l++) {
      const int wb = 32 * (grp / 2) + l;
      const unsigned byte = ub[((wb / 16) * 32 + lane) * 16 + wb % 16];
      const unsigned code = (grp % 2) == 0 ? (byte & 0xF) : (byte >> 4);
      dot += (int)code * codes[s * 256 + 32 * grp + l];
    }
  } else {
    const size_t s = g / 16;
    const int grp = (int)(g % 16);
    const uint8_t *ub = slot_unit(geo, type, row, s, lane);
    for (int l16 = 0; l16 < 16; l16++) {
      const int p = 16 * grp + l16;
      const int n = p / 128, r = p % 128, quarter = r / 32, l = r % 32;
      const int qlb = 64 * n + l + ((quarter & 1) ? 32 : 0), qhb = 128 + 32 * n + l;
      const unsigned qlv = ub[((qlb / 16) * 32 + lane) * 16 + qlb % 16];
      const unsigned qhv = ub[((qhb / 16) * 32 + lane) * 16 + qhb % 16];
      const unsigned lo = quarter < 2 ? (qlv & 0xF) : (qlv >> 4);
      const int code = (int)(lo | (((qhv >> (2 * quarter)) & 3) << 4)) - 32;
      dot += code * codes[s * 256 + p];
    }
  }
  dots[idx] = dot;
}

// ---- host side: planning, repack, launches ---------------------------------------------------

size_t packed_bytes(const GemvPlan &pl, uint32_t type) {
  return pl.n_rt * (size_t)pl.units * (size_t)unit_bytes_of(type);
}

cudaError_t launch_repack(const GemvPlan &pl, const uint8_t *d_raw, uint8_t *d_pack,
                          uint32_t type, size_t n_out, size_t n_in, size_t row_bytes,
                          cudaStream_t stream) {
  const int kslots = units_per_row_tile(type, n_in);
  const int nblk = type == kQ8_0 ? (int)((n_in + 31) / 32) : kslots;
  const size_t total = packed_bytes(pl, type);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  size_t blocks = (total + threads - 1) / threads;
  if (blocks > 65535u * 16u) blocks = 65535u * 16u;
  repack_kernel<<<(unsigned)blocks, threads, 0, stream>>>(d_raw, d_pack, type, n_out, row_bytes,
                                                          pl.units, pl.L, kslots, nblk, total);
  return cudaGetLastError();
}

cudaError_t launch_block_dots(const GemvPlan &pl, uint32_t type, const uint8_t *pack,
                              size_t n_out, size_t n_in, const int8_t *codes, int32_t *dots,
                              cudaStream_t stream) {
  const int kslots = units_per_row_tile(type, n_in);
  const size_t per_row =
      type == kQ8_0 ? (n_in + 31) / 32 : (size_t)kslots * (type == kQ6_K ? 16 : 8);
  const size_t total = n_out * per_row;
  if (total == 0) return cudaSuccess;
  block_dots_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
      type, PackGeo{pack, pl.units, pl.L}, n_out, per_row, codes, dots);
  return cudaGetLastError();
}

static size_t warp_act_bytes(uint32_t t) {
  return t == kQ8_0 ? sizeof(WarpAct<kQ8_0>)
                    : (t == kQ4_K ? sizeof(WarpAct<kQ4_K>) : sizeof(WarpAct<kQ6_K>));
}

// The most CTAs of a K split that run as one cluster (8, the portable cluster size).
static int max_cluster_split() {
  static const int v = [] {
    const char *e = std::getenv("APX_GEMV_CLUSTER_MAX");  // 0 or 1: scratch splits only
    return e ? std::max(0, std::min(8, atoi(e))) : 8;
  }();
  return v;
}

GemvPlan plan_gemv(uint32_t type, size_t n_out, size_t n_in, int sm_count) {
  GemvPlan pl{};
  const int K = units_per_row_tile(type, n_in);  // K-slots per row (0 for n_in = 0)
  // up to two resident waves of one unit per warp: past that the persistent streaming kernel;
  // below it the streaming kernel's per-warp chunks would be too short to amortise its flush
  const size_t wave = (size_t)sm_count * 48;
  const size_t T1 = (n_out + 31) / 32 * (size_t)K;
  if (T1 > wave) {
    // persistent streaming kernel: 2 CTAs of 8 warps per SM, one contiguous chunk per warp
    pl.pipe = true;
    pl.L = 1;
    pl.units = K;
    pl.n_rt = (n_out + 31) / 32;
    const int span = type == kQ8_0 ? 128 : 256;
    const size_t nel = (size_t)K * span;
    pl.smem = nel + ((nel / 32 + 3) & ~(size_t)3) * 4 + nel / 16 * 8;
    const int per_sm = type != kQ6_K && pl.smem * 2 <= 200 * 1024 ? 2 : 1;
    pl.block = type == kQ6_K ? 384 : 256;
    pl.grid = (unsigned)(sm_count * per_sm);
    const long long V = (long long)pl.grid * (pl.block / 32);
    pl.chunk = (long long)((T1 + V - 1) / V);
    pl.kmax = (int)((K + pl.chunk - 1) / pl.chunk) + 1;
    pl.R = pl.P = pl.ksplit = 1;
    return pl;
  }
  // One wave: one unit per warp, every load in flight at once.  Few, long rows spread
  // their K-slots over 2 or 4 lanes so a row tile's units fit one CTA.
  pl.pipe = false;
  pl.L = 1;
  while (pl.L < 4 && (K + pl.L - 1) / pl.L > 12) pl.L *= 2;
  // More row tiles than SMs whose units are too many for two to share a CTA would stack two
  // CTAs of the launch on a few SMs (their late start is the launch's tail): then 2L lanes a
  // row, when that gives one CTA per SM with an even share of row tiles.  Q8_0 4864x896
  // (configs[0]): 152 CTAs of 7 warps 2.68 us, 148 CTAs of 3 row tiles x 4 warps 2.44 us.
  auto shared_fit = [&](int L, bool &fits) {
    const size_t u = (size_t)(K + L - 1) / L, rt = (n_out + 32 / L - 1) / (32 / L);
    const size_t share = (rt + sm_count - 1) / sm_count;
    fits = share * u <= 12;
    return u <= 12 && rt > (size_t)sm_count;
  };
  for (bool fits = false; pl.L < 4 && shared_fit(pl.L, fits) && !fits;) {
    bool fits2 = false;
    if (!shared_fit(2 * pl.L, fits2) || !fits2) break;
    pl.L *= 2;
  }
  const int H = 32 / pl.L;
  const int U = (K + pl.L - 1) / pl.L;
  const size_t n_rt = (n_out + H - 1) / H;
  pl.units = U;
  pl.n_rt = n_rt;
  const int w = std::max(1, U);
  if (w <= 12) {
    pl.ksplit = 1;
    pl.P = w;
    // More row tiles than SMs: one CTA per SM with an even share of them (1 or 2 here), when
    // the share fits 12 warps.  A CTA then fills half an SM's registers, so exactly one CTA of
    // this projection and one of the next (programmatic dependent launch) sit on every SM,
    // and the block scheduler cannot stack several CTAs of one launch on one SM.
    const size_t share = (n_rt + sm_count - 1) / sm_count;
    pl.R = n_rt > (size_t)sm_count && share * pl.P <= 12 ? (int)share : 1;
  } else {
    pl.ksplit = (w + 11) / 12;
    pl.P = (w + pl.ksplit - 1) / pl.ksplit;
    pl.R = 1;
  }
  if ((size_t)pl.R > n_rt) pl.R = (int)(n_rt ? n_rt : 1);
  const size_t rows = pl.R > 1 ? (size_t)sm_count : (n_rt + pl.R - 1) / pl.R;
  // A K split of up to 8 CTAs runs as one thread-block cluster per row tile: the partial sums
  // meet in CTA 0's shared memory instead of global scratch and an arrival counter.  (Splitting
  // row tiles over clusters only to even out the CTAs per SM was slower on the configs[0] and
  // configs[1] shapes: 608 CTAs of 2 warps 3.08 us against 152 of 7 warps 2.69 us.)
  pl.cluster = pl.ksplit > 1 && pl.ksplit <= max_cluster_split() ? pl.ksplit : 0;
  pl.grid = (unsigned)(rows * pl.ksplit);
  pl.block = 32 * pl.R * pl.P;
  const size_t stage = (size_t)pl.R * pl.P * warp_act_bytes(type);
  const size_t red = (size_t)pl.R * pl.P * 32 * sizeof(Acc128) + 64;
  pl.act_bytes = (int)((std::max(stage, red) + 15) & ~(size_t)15);
  // a cluster's partial sums: [ksplit][32] in CTA 0's shared memory, after the staging
  pl.w_off = (int)((pl.act_bytes + (pl.cluster ? (size_t)pl.cluster * 32 * sizeof(Acc128) : 0) +
                    15) & ~(size_t)15);
  // Weights in registers while every CTA is resident at once at 80 registers a thread (25 warps
  // an SM); otherwise in shared memory at 64 (32 warps), e.g. 448 CTAs of 8 warps (3584x8192
  // Q4_K): 7.0 -> 5.4 us.  Measured the other way on the configs[0]/[1] shapes, which fit:
  // 2.58 -> 2.86 us (8960x1536), 3.70 -> 4.55 us (1536x8960): smaller CTAs let the block
  // scheduler stack two of one launch on an SM.
  const int per_sm80 = std::max(1, 25 / (pl.R * pl.P));
  pl.smem_w = pl.grid > (unsigned)sm_count * (unsigned)per_sm80;
  pl.smem = pl.w_off + (pl.smem_w ? (size_t)pl.R * pl.P * unit_bytes_of(type) : 0);
  return pl;
}

size_t gemv_scratch_bytes(const GemvPlan &pl) {
  if (pl.pipe) return pl.n_rt * (size_t)pl.kmax * 32 * sizeof(Acc128) + pl.n_rt * sizeof(unsigned);
  if (pl.ksplit <= 1 || pl.cluster > 1) return 0;
  return pl.n_rt * (size_t)pl.ksplit * 32 * sizeof(Acc128) + pl.n_rt * sizeof(unsigned);
}

// Programmatic dependent launch is on unless APX_PDL=0 in the environment (read once).
static bool pdl_enabled() {
  static const bool on = [] {
    const char *v = std::getenv("APX_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Set while a launch is captured behind a copy (a graph edge from a copy node cannot be
// programmatic): launches from this thread then go without the attribute.
static thread_local bool tl_pdl_suppressed = false;
void set_pdl_suppressed(bool on) { tl_pdl_suppressed = on; }
bool pdl_allowed() { return pdl_enabled() && !tl_pdl_suppressed; }

template <typename Kern, typename Args>
static cudaError_t launch_cfg(Kern kern, const GemvPlan &pl, const Args &a, cudaStream_t stream) {
  if (pl.smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)pl.smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(pl.block);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled() && !tl_pdl_suppressed) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  if (!pl.pipe && pl.cluster > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)pl.cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    n++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

cudaError_t launch_gemv(const GemvPlan &pl, uint32_t type, const uint8_t *pack, void *scratch,
                        size_t n_out, size_t n_in, const int8_t *codes, const uint8_t *exps,
                        const void *desc, long long *out_q32, float *out_f32,
                        unsigned long long *status, cudaStream_t stream, const PeerRows *peers) {
  const PeerRows no_peers{};
  if (n_out == 0) return cudaSuccess;
  if ((pl.pipe || (pl.ksplit > 1 && pl.cluster <= 1)) && !scratch) return cudaErrorInvalidValue;
  if (pl.units > 0 && !pack) return cudaErrorInvalidValue;  // a plan that reads no payload
  if (pl.pipe) {
    StreamArgs sa;
    sa.pack = pack;
    sa.units = pl.units;
    sa.n_rt = pl.n_rt;
    sa.n_out = n_out;
    sa.n_in = n_in;
    sa.codes = codes;
    sa.exps = exps;
    sa.desc = reinterpret_cast<const ActDesc *>(desc);
    sa.out_q32 = out_q32;
    sa.out_f32 = out_f32;
    sa.status = status;
    sa.partials = reinterpret_cast<Acc128 *>(scratch);
    sa.counters = reinterpret_cast<unsigned *>(reinterpret_cast<Acc128 *>(scratch) +
                                               pl.n_rt * (size_t)pl.kmax * 32);
    sa.chunk = pl.chunk;
    sa.kmax = pl.kmax;
    sa.peers = peers ? *peers : no_peers;
    switch (type) {
      case kQ8_0: return launch_cfg(gemv_stream_kernel<kQ8_0>, pl, sa, stream);
      case kQ4_K: return launch_cfg(gemv_stream_kernel<kQ4_K>, pl, sa, stream);
      case kQ6_K: return launch_cfg(gemv_stream_kernel<kQ6_K>, pl, sa, stream);
      default: return cudaErrorInvalidValue;
    }
  }
  GemvArgs a;
  a.pack = pack;
  a.units = pl.units;
  a.L = pl.L;
  a.n_rt = pl.n_rt;
  a.n_out = n_out;
  a.n_in = n_in;
  a.codes = codes;
  a.exps = exps;
  a.desc = reinterpret_cast<const ActDesc *>(desc);
  a.out_q32 = out_q32;
  a.out_f32 = out_f32;
  a.status = status;
  const bool global_split = pl.ksplit > 1 && pl.cluster <= 1;
  a.partials = global_split ? reinterpret_cast<Acc128 *>(scratch) : nullptr;
  a.counters = global_split ? reinterpret_cast<unsigned *>(reinterpret_cast<Acc128 *>(scratch) +
                                                           pl.n_rt * pl.ksplit * 32)
                            : nullptr;
  a.R = pl.R;
  a.P = pl.P;
  a.ksplit = pl.ksplit;
  a.cluster = pl.cluster > 1 ? pl.cluster : 1;
  a.act_bytes = pl.act_bytes;
  a.w_off = pl.w_off;
  a.peers = peers ? *peers : no_peers;
  a.grp = GemvGroup{};
  switch (type) {
    case kQ8_0:
      return pl.smem_w ? launch_cfg(gemv_kernel_smem<kQ8_0>, pl, a, stream)
                       : launch_cfg(gemv_kernel<kQ8_0>, pl, a, stream);
    case kQ4_K:
      return pl.smem_w ? launch_cfg(gemv_kernel_smem<kQ4_K>, pl, a, stream)
                       : launch_cfg(gemv_kernel<kQ4_K>, pl, a, stream);
    case kQ6_K:
      return pl.smem_w ? launch_cfg(gemv_kernel_smem<kQ6_K>, pl, a, stream)
                       : launch_cfg(gemv_kernel<kQ6_K>, pl, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_gemv_group(const GemvPlan &pl, uint32_t type, const GemvGroup &grp,
                              size_t n_in, const int8_t *codes, const uint8_t *exps,
                              const void *desc, cudaStream_t stream) {
  if (grp.n < 1 || grp.n > kMaxGroup || pl.pipe || (pl.ksplit != 1 && pl.cluster != pl.ksplit))
    return cudaErrorInvalidValue;  // a K split only through a cluster: no scratch here
  GemvArgs a{};
  a.pack = grp.pack[0];
  a.units = pl.units;
  a.L = pl.L;
  a.n_rt = pl.n_rt;
  a.n_out = grp.n_out[0];
  a.n_in = n_in;
  a.codes = codes;
  a.exps = exps;
  a.desc = reinterpret_cast<const ActDesc *>(desc);
  a.out_q32 = grp.out_q32[0];
  a.out_f32 = grp.out_f32[0];
  a.status = grp.status[0];
  a.R = pl.R;
  a.P = pl.P;
  a.ksplit = pl.ksplit;
  a.cluster = pl.cluster > 1 ? pl.cluster : 1;
  a.act_bytes = pl.act_bytes;
  a.w_off = pl.w_off;
  a.grp = grp;
  switch (type) {
    case kQ8_0:
      return pl.smem_w ? launch_cfg(gemv_kernel_smem<kQ8_0>, pl, a, stream)
                       : launch_cfg(gemv_kernel<kQ8_0>, pl, a, stream);
    case kQ4_K:
      return pl.smem_w ? launch_cfg(gemv_kernel_smem<kQ4_K>, pl, a, stream)
                       : launch_cfg(gemv_kernel<kQ4_K>, pl, a, stream);
    case kQ6_K:
      return pl.smem_w ? launch_cfg(gemv_kernel_smem<kQ6_K>, pl, a, stream)
                       : launch_cfg(gemv_kernel<kQ6_K>, pl, a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace apx
