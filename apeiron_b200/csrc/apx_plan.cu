// apx_plan.cu — the projections of a decode step in one persistent launch.
//
// A plan lists projections (a tensor, its activation, its outputs) in dependency order, and
// optionally FFNs: a gate and an up projection of one activation whose finish runs SwiGLU and
// quant_act (the SwiGLU and quantization stages of fused_ffn_task,
// src/engine/chart/ffn.rs:1577-1594) into an activation a later projection reads (down).  One
// launch of a persistent grid runs the whole list; each projection's outputs, refusals and
// rounding are those of apx_matvec_async on the same inputs (matvec_q8act,
// chart/mod.rs:1887-1925), each FFN's those of apx_swiglu_quant_async.
//
// Work.  Every projection's row tiles are cut into pieces of at most kPlanPiece units of the
// tensor's repacked layout (fewer for a short plan); the pieces of all projections form one
// queue.  Warp v of the V in the grid starts on piece v; every later piece is taken from a shared
// counter, one piece ahead (while the warp folds its current piece, the next one's weights
// stream in behind it), so warps that draw short pieces take more of them.  A warp streams its
// pieces' units through a ring in shared memory (1D bulk copies, one unit in flight while one
// folds; the first piece's copies start before the wait for the previous kernel) and folds each
// exactly as the one-wave GEMV kernel does; a row tile of one piece finishes in the warp, a row
// tile of several through partial sums in the plan's scratch and a self-resetting arrival counter
// (the last to arrive finishes it).
//
// Hand-off.  An FFN's gate and up run as one paired record: a piece alternates gate and up units
// over one staged activation chunk, so the warp that finishes a row tile holds both projections'
// rows.  When a row tile is a whole 32-row block of h (one quant_act block, L = 1) that warp runs
// the block's SwiGLU under the carrier and quant_act at once; otherwise the block's row tiles
// count in on its counter and the last runs it.  The last block of the FFN computes the
// descriptor from the blocks' exponent bytes and raises the FFN's flag.  A warp whose piece reads
// that activation waits on the flag before it takes its next piece, with a bound (about one
// second) after which the projection refuses with APX_ERR_DEVICE_TIMEOUT.  The host queues
// projections by dependency level, an FFN's producers ahead of the level's other work and its
// readers in the next level, so the flag is usually up when a warp gets there.  Every wait ends:
// pieces are taken in queue order, a warp holds at most its current piece and the one after it,
// and it waits only for its current piece, before taking the next; every piece a wait depends
// on sits earlier in the queue, so by induction on queue position each piece's holder reaches
// it (its current piece is earlier and completes) and its producers complete, the grid being
// co-resident.  The last CTA out resets the counters and flags for the next launch.
#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

#include "apx_common.cuh"
#include "apx_kernels.h"
#include "apx_pack.cuh"
#include "apx_quant.cuh"
#include "apx_swiglu.cuh"
#include "apx_unit.cuh"

namespace apx {

namespace {

constexpr int kPlanPiece = 8;  // units per piece at most

struct PlanProjD {
  const uint8_t *pack;
  long long *out_q32;
  float *out_f32;
  unsigned long long *status;
  Acc128 *part;   // [n_rt][npieces][1 + paired][32] when npieces > 1
  unsigned *cnt;  // [n_rt] arrivals (self-resetting) when npieces > 1
  size_t n_out, n_in;
  int n_rt, U, L, plen, npieces, piece0;
  int act, ffn;  // activation read; FFN fed (-1 for none)
  // An FFN's gate and up as one record (paired = 1): a piece streams gate unit u (pack) and
  // up unit u (pack2) in turn over one staged activation chunk, and the warp that finishes a
  // row tile holds both outputs of its 32-row block of h, so it runs the block's SwiGLU at
  // once.  Virtual unit 2u + 0 / 1 is gate / up unit u.
  int paired;
  const uint8_t *pack2;
  long long *out2_q32;
  float *out2_f32;
  unsigned long long *status2;
};

struct PlanActD {
  const int8_t *codes;
  const uint8_t *exps;
  const ActDesc *desc;
  int ffn;  // the FFN of this launch that writes it, or -1 (ready when the launch starts)
  int pad;
};

struct PlanFfnD {
  const long long *gate, *up;  // the gate and up projections' Q32.32 outputs
  const unsigned long long *gate_status, *up_status;
  long long *h;  // or null
  int8_t *codes;
  uint8_t *exps;
  ActDesc *desc;
  unsigned long long *status;  // the first refusing SwiGLU lane
  unsigned *pair;              // [n_rt] row tiles of the block done (self-resetting)
  size_t n;
  int n_rt, carrier, refused;  // refused: a non-finite weight row below n (found at upload)
  int n_peers;                 // row shards: where else the blocks and the descriptor go
  int8_t *peer_codes[7];
  uint8_t *peer_exps[7];
  ActDesc *peer_desc[7];
};

struct PlanArgs {
  const PlanProjD *proj;
  const PlanActD *act;
  const PlanFfnD *ffn;
  PlanCtl *ctl;
  int n_proj, n_ffn, total, V;
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct Piece {
  int j, rt, q, u0, u1;
};

__device__ __forceinline__ Piece decode_piece(const PlanArgs &g, const int *p0, int x) {
  int lo = 0, hi = g.n_proj - 1;  // the last projection whose first piece is <= x
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (p0[mid] <= x) lo = mid;
    else hi = mid - 1;
  }
  const PlanProjD &P = g.proj[lo];
  const int local = x - p0[lo], np = P.npieces, plen = P.plen;
  Piece pc;
  pc.j = lo;
  pc.rt = local / np;
  pc.q = local % np;
  pc.u0 = (pc.q * plen) << P.paired;  // virtual units: 2u + 0 / 1 in a paired record
  pc.u1 = min(P.U, pc.q * plen + plen) << P.paired;
  return pc;
}

// The weights of (virtual) unit u of row tile rt.
template <uint32_t T>
__device__ __forceinline__ const uint8_t *unit_ptr(const PlanProjD &P, int rt, int u) {
  const uint8_t *pk = P.paired && (u & 1) ? P.pack2 : P.pack;
  return pk + ((size_t)rt * P.U + (u >> P.paired)) * (size_t)Fam<T>::unit_bytes;
}

// SwiGLU + quant_act of block rt of FFN f (lane = row), its statistics, and — for the last
// block — the descriptor and the flag.  Mirrors swiglu_quant_kernel and ffn_desc_kernel.
__device__ void ffn_block(const PlanArgs &g, int f, int rt, int lane) {
  const PlanFfnD &F = g.ffn[f];
  const size_t row = (size_t)rt * 32 + lane;
  long long v = 0;
  bool ok = true;
  if (row < F.n) {
    const int rc = swiglu_dev(__ldcg(F.gate + row), __ldcg(F.up + row), F.carrier, v);
    if (rc) {
      ok = false;
      v = 0;
      atomicMin(F.status, pack_status(row, APX_ERR_SWIGLU_REFUSED, (unsigned)rc));
    }
    if (F.h) F.h[row] = v;
  }
  unsigned long long mx = uabs64(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xFFFFFFFFu, mx, o);
    mx = t > mx ? t : mx;
  }
  const int e = act_scale_exp(mx);
  int w_status = __any_sync(0xFFFFFFFFu, !ok) ? (int)APX_ERR_QUANT_REFUSED : (int)APX_OK;
  int code = 0;
  if (e == 99) {
    w_status = APX_ERR_QUANT_REFUSED;
  } else if (e >= 0) {
    const unsigned long long m = uabs64(v);
    const unsigned long long S = 1ull << e, qq = m >> e, r = m & (S - 1);
    const unsigned long long mag = qq + (2 * r >= S ? 1ull : 0ull);
    code = v < 0 ? -(int)mag : (int)mag;
    if (__any_sync(0xFFFFFFFFu, mag > 127 || !product_fits(code, e)))
      w_status = APX_ERR_QUANT_REFUSED;
  }
  const uint8_t eb = e < 0 || e == 99 ? (uint8_t)APX_EXP_ZERO : (uint8_t)e;
  if (row < F.n) F.codes[row] = (int8_t)code;
  if (lane == 0) F.exps[rt] = eb;
#pragma unroll 1
  for (int p = 0; p < F.n_peers; p++) {  // row shards: the block into the other ranks' buffers
    if (row < F.n) F.peer_codes[p][row] = (int8_t)code;
    if (lane == 0) F.peer_exps[p][rt] = eb;
  }
  // A refusal is rare: one atomic on the FFN's status word then.  The exponent statistics are
  // not counted per block: the last block reads every block's exponent byte instead.
  // Hand-offs through a counter: the lanes' stores, __syncwarp, then lane 0's release fence
  // and relaxed atomic; the last arrival's lane 0 fences (acquire) before __syncwarp and the
  // lanes' loads.
  int *st = g.ctl->stats[f];
  if (lane == 0 && w_status != APX_OK) atomicMax(st + 2, w_status);
  __syncwarp();
  fence_acq_rel_gpu();  // every lane's stores (and the refusal) before the block counts
  unsigned done = 0;
  if (lane == 0) done = atomicAdd(&g.ctl->ready[f], 1u);
  done = __shfl_sync(0xFFFFFFFFu, done, 0);
  if (done != (unsigned)F.n_rt - 1) return;
  // every block is in: every row tile of gate and up has finished (its outputs and its refusals
  // were stored before its count), so their status words are final too
  fence_acq_rel_gpu();
  __syncwarp();
  int emin = 1 << 30, emax = -1;
  unsigned nz = 0;
  for (int b = lane; b < F.n_rt; b += 32) {
    const unsigned eb = __ldcg(F.exps + b);
    if (eb != APX_EXP_ZERO) {
      emin = min(emin, (int)eb);
      emax = max(emax, (int)eb);
      nz++;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    emin = min(emin, __shfl_xor_sync(0xFFFFFFFFu, emin, o));
    emax = max(emax, __shfl_xor_sync(0xFFFFFFFFu, emax, o));
    nz += __shfl_xor_sync(0xFFFFFFFFu, nz, o);
  }
  if (lane == 0) {
    int status = __ldcg(st + 2);
    if (F.refused || __ldcg(F.gate_status) != ~0ull || __ldcg(F.up_status) != ~0ull)
      status = max(status, (int)APX_ERR_QUANT_REFUSED);  // h is undefined where they refused
    ActDesc d;
    d.status = status;
    d.emax = emax;
    d.emin = emax >= 0 ? emin : 0;
    d.n_in = (int32_t)F.n;
    d.nz = nz;
    d.pad[0] = 0;  // quant_act codes are never -128
    d.pad[1] = 0;
    d.pad[2] = 0;
    *F.desc = d;
    for (int p = 0; p < F.n_peers; p++) *F.peer_desc[p] = d;
    fence_acq_rel_gpu();
    atomicExch(&g.ctl->flag[f], 1u);
  }
}

// Wait for FFN f's descriptor: about one second at most, and none at all once a wait of this
// launch has given up (the launch's later readers then refuse at once).
__device__ __forceinline__ bool wait_flag(const PlanArgs &g, int f) {
  if (ld_acquire(&g.ctl->flag[f])) return true;
  unsigned long long t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (int it = 0; it < kWaitLimit; it++) {
    __nanosleep(128);
    if (ld_acquire(&g.ctl->flag[f])) return true;
    if ((it & 15) == 15) {
      if (ld_acquire(&g.ctl->abort)) return false;
      unsigned long long now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (now - t0 > 1000000000ull) break;
    }
  }
  atomicExch(&g.ctl->abort, 1u);
  return false;
}

// Launch shape per family: warps per CTA, CTAs per SM, weight ring slots per warp.  Each warp
// streams its units through a ring of kSlots unit buffers in shared memory, filled by 1D bulk
// copies (cp.async.bulk, no multicast) that complete on one mbarrier per slot: kSlots - 1 units
// in flight while one folds.  Measured on B200 over a decode step's 168 projections: sixteen
// warps per SM with two slots each beat twelve with three (the fold is issue-bound: warps hide
// its latency better than deeper rings hide HBM's) and eight or six with five or seven slots.
template <uint32_t T>
struct PlanShape {
  static constexpr int kWarps = 8;
  static constexpr int kCtas = T == kQ6_K ? 1 : 2;
  static constexpr int kSlots = T == kQ6_K ? 3 : 2;
  static constexpr int kUnit = Fam<T>::unit_bytes;
  static constexpr int kThreads = 32 * kWarps;
  static_assert(kUnit % 16 == 0, "bulk copies move whole 16-byte chunks");
};

template <uint32_t T>
__host__ __device__ constexpr size_t plan_ring_bytes() {
  return (size_t)PlanShape<T>::kWarps * PlanShape<T>::kSlots * PlanShape<T>::kUnit;
}
template <uint32_t T>
__host__ __device__ constexpr size_t plan_fixed_smem() {  // ring, barriers, activation slots
  return plan_ring_bytes<T>() + (size_t)PlanShape<T>::kWarps * PlanShape<T>::kSlots * 8 +
         (size_t)2 * PlanShape<T>::kWarps * sizeof(WarpAct<T>);
}

// The order-fence between this thread's reads of a ring slot and the bulk copy that refills it.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One warp's stream of units: the units of its current piece, then those of the piece it took
// next.  k_issue / k_fold count units copied / folded; unit k sits in slot k % kSlots, and its
// copy completes phase (k / kSlots) & 1 of that slot's barrier.
template <uint32_t T>
struct UnitStream {
  uint8_t *ring;   // this warp's kSlots buffers
  uint64_t *bars;  // their barriers
  int k_issue, k_fold;
  int nxt_on;      // the issue cursor is in the next piece
  int iu;          // the issue cursor's unit

  // Copy units ahead while slots are free: the rest of `pc`, then `pn` when it exists.
  __device__ __forceinline__ void top_up(const PlanArgs &g, const Piece &pc, const Piece &pn,
                                         bool have_next, int lane) {
    constexpr int S = PlanShape<T>::kSlots;
    while (k_issue - k_fold < S) {
      const Piece &p = nxt_on ? pn : pc;
      if (iu >= p.u1) {
        if (nxt_on || !have_next) break;
        nxt_on = 1;
        iu = pn.u0;
        continue;
      }
      if (lane == 0) {
        const int s = k_issue % S;
        mbar_expect_tx(bars + s, PlanShape<T>::kUnit);
        bulk_g2s(ring + (size_t)s * PlanShape<T>::kUnit, unit_ptr<T>(g.proj[p.j], p.rt, iu),
                 PlanShape<T>::kUnit, bars + s);
      }
      iu++;
      k_issue++;
    }
  }

  // The next unit's slot, once its copy has landed (bounded: false when the wait gave up).
  __device__ __forceinline__ bool wait_front(uint8_t *&slot) {
    constexpr int S = PlanShape<T>::kSlots;
    const int s = k_fold % S;
    slot = ring + (size_t)s * PlanShape<T>::kUnit;
    return mbar_wait(bars + s, (uint32_t)((k_fold / S) & 1));
  }

  // Hand the front slot back after the warp read it: the next copy may refill it.
  __device__ __forceinline__ void release_front() {
    fence_proxy_async();
    __syncwarp();
    k_fold++;
  }

  // The piece the stream moves on to: the issue cursor leaves the finished piece.
  __device__ __forceinline__ void advance(const Piece &next) {
    if (nxt_on) {
      nxt_on = 0;
    } else {
      iu = next.u0;
    }
  }
};

template <uint32_t T>
__global__ void __launch_bounds__(PlanShape<T>::kThreads, PlanShape<T>::kCtas)
    plan_kernel(PlanArgs g) {
  using F = Fam<T>;
  using SH = PlanShape<T>;
  extern __shared__ __align__(128) unsigned char smem[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + plan_ring_bytes<T>()) + warp * SH::kSlots;
  WarpAct<T> *wa = reinterpret_cast<WarpAct<T> *>(smem + plan_ring_bytes<T>() +
                                                  (size_t)SH::kWarps * SH::kSlots * 8) +
                   2 * warp;
  int *s_p0 = reinterpret_cast<int *>(smem + plan_fixed_smem<T>());
  for (int i = threadIdx.x; i < g.n_proj; i += blockDim.x) s_p0[i] = g.proj[i].piece0;
  if (lane == 0)
    for (int s = 0; s < SH::kSlots; s++) mbar_init(bars + s, 1);
  __syncthreads();
  // the first pieces go one per CTA before any CTA takes a second, so a short plan spreads
  // over every SM
  const int v = warp * (int)gridDim.x + (int)blockIdx.x;

  pdl_launch_dependents();
  UnitStream<T> us{smem + (size_t)warp * SH::kSlots * SH::kUnit, bars, 0, 0, 0, 0};
  int x = v < g.total ? v : -1;
  Piece pc{0, 0, 0, 0, 0}, pn{0, 0, 0, 0, 0};
  if (x >= 0) {  // the first piece is static: its weights stream in before the wait
    pc = decode_piece(g, s_p0, x);
    us.iu = pc.u0;
    us.top_up(g, pc, pn, false, lane);
  }
  pdl_wait();

  const Chunk zero_chunk{make_uint4(0, 0, 0, 0), APX_EXP_ZERO};
  auto fetch = [&](const PlanProjD &Q, const PlanActD &B, int u, Chunk &a0, Chunk &a1) {
    const int nq = Q.L * F::span / 16;
    a0 = zero_chunk;
    a1 = zero_chunk;
    if (B.ffn >= 0) {
      if (lane < nq) a0 = load_chunk_cg(B.codes, B.exps, Q.n_in, chunk_first<T>(u, Q.L, lane));
      if (lane + 32 < nq)
        a1 = load_chunk_cg(B.codes, B.exps, Q.n_in, chunk_first<T>(u, Q.L, lane + 32));
    } else {
      if (lane < nq) a0 = load_chunk(B.codes, B.exps, Q.n_in, chunk_first<T>(u, Q.L, lane));
      if (lane + 32 < nq)
        a1 = load_chunk(B.codes, B.exps, Q.n_in, chunk_first<T>(u, Q.L, lane + 32));
    }
  };
  Chunk c0 = zero_chunk, c1 = zero_chunk;
  bool act_pre = false;  // c0/c1 already hold the current piece's first activation chunk

  while (x >= 0) {
    const PlanProjD &P = g.proj[pc.j];
    const int L = P.L, H = 32 / L, slot = lane % L;
    const int nch = L * F::span / 16;
    const PlanActD &A = g.act[P.act];
    const bool produced = A.ffn >= 0;
    bool ready = true;
    if (produced) {  // before taking the next piece: a waiting warp holds no later work
      int r = 1;
      if (lane == 0) r = wait_flag(g, A.ffn) ? 1 : 0;
      ready = __shfl_sync(0xFFFFFFFFu, r, 0) != 0;
      __syncwarp();  // every lane's reads of the activation come after the acquire
    }
    ActDesc desc;
    if (produced) {
      const int4 d0 = __ldcg(reinterpret_cast<const int4 *>(A.desc));
      const int4 d1 = __ldcg(reinterpret_cast<const int4 *>(A.desc) + 1);
      memcpy(&desc, &d0, 16);
      memcpy(reinterpret_cast<char *>(&desc) + 16, &d1, 16);
    } else {
      desc = *A.desc;
    }
    // the next piece, taken now (after this piece's wait): its weights follow this piece's
    // through the ring
    unsigned nxq = 0;
    if (lane == 0) nxq = (unsigned)g.V + atomicAdd(&g.ctl->queue, 1u);
    nxq = __shfl_sync(0xFFFFFFFFu, nxq, 0);
    const int xn = nxq < (unsigned)g.total ? (int)nxq : -1;
    if (xn >= 0) pn = decode_piece(g, s_p0, xn);
    us.top_up(g, pc, pn, xn >= 0, lane);

    // the fold: the fast one within the family's spread limit, the wide one beyond it while
    // the call bound holds; other activations take the checked rows
    const bool ok = ready && desc.status == APX_OK;
    const bool narrow = ok && fast_path<T>(desc, P.n_in);
    const bool wide = ok && !narrow && wide_path<T>(desc, P.n_in);
    const bool fast = narrow || wide;
    const int sh = P.paired;  // units alternate gate, up: one activation chunk serves two
    if (fast && !act_pre) fetch(P, A, pc.u0 >> sh, c0, c1);
    bool next_pre = false, copies_ok = true;
    Acc128 acc, acc2;  // acc2: the up projection's sums in a paired record
    acc_zero(acc);
    acc_zero(acc2);
    for (int u = pc.u0; u < pc.u1; u++) {
      uint8_t *sl;
      const bool got = us.wait_front(sl);
      copies_ok = copies_ok && got;
      if (!fast) {  // the slot is consumed all the same
        us.release_front();
        us.top_up(g, pc, pn, xn >= 0, lane);
        continue;
      }
      const int ru = u >> sh;               // the real unit
      const bool second = sh && (u & 1);     // up's unit u, over the chunk gate's staged
      WarpAct<T> &wb = wa[ru & 1];
      if (!second) {
        store_chunk<T>(wb, c0, lane, lane < nch, desc.emin, wide);
        if (nch > 32) store_chunk<T>(wb, c1, lane + 32, lane + 32 < nch, desc.emin, wide);
        __syncwarp();
        if (ru + 1 < (pc.u1 >> sh)) {
          fetch(P, A, ru + 1, c0, c1);
        } else if (xn >= 0) {  // the next piece's first chunk, when its activation is ready now
          const PlanProjD &Q = g.proj[pn.j];
          const PlanActD &B = g.act[Q.act];
          int r = 1;
          if (B.ffn >= 0 && lane == 0) r = ld_acquire(&g.ctl->flag[B.ffn]) ? 1 : 0;
          r = __shfl_sync(0xFFFFFFFFu, r, 0);
          __syncwarp();
          if (r) {
            fetch(Q, B, pn.u0 >> Q.paired, c0, c1);
            next_pre = true;
          }
        }
      }
      Acc128 t;
      acc_zero(t);
      fold_unit_smem<T>(t, sl, lane, wb.codes + slot * slot_ints<T>(),
                        wb.e + slot * (F::span / 32), wb.xs + slot * F::nxs, desc.emin, wide);
      if (second) acc_add(acc2, t);
      else acc_add(acc, t);
      us.release_front();  // the fold has read the slot: the next copy may refill it
      us.top_up(g, pc, pn, xn >= 0, lane);
    }
    const bool lead = pc.q == 0;  // the piece that speaks for its row tile off the fast path
    bool done = false;            // this warp completed the row tile
    if (!copies_ok) {             // a weight copy did not land in time
      if (lane == 0) {
        atomicExch(&g.ctl->abort, 1u);
        atomicMin(P.status, pack_status(0, APX_ERR_DEVICE_TIMEOUT, 0));
        if (sh) atomicMin(P.status2, pack_status(0, APX_ERR_DEVICE_TIMEOUT, 0));
      }
      done = lead;
    } else if (!ready) {
      if (lead && lane == 0) {
        atomicMin(P.status, pack_status(0, APX_ERR_DEVICE_TIMEOUT, 0));
        if (sh) atomicMin(P.status2, pack_status(0, APX_ERR_DEVICE_TIMEOUT, 0));
      }
      done = lead;
    } else if (desc.status != APX_OK) {  // the activation is refused (chart/mod.rs:1904-1907)
      if (lead && pc.rt == 0 && lane == 0) {
        atomicMin(P.status, pack_status(0, (unsigned)desc.status, 0));
        if (sh) atomicMin(P.status2, pack_status(0, (unsigned)desc.status, 0));
      }
      done = lead;
    } else if (!fast) {
      if (lead && slot == 0) {
        checked_row<T>(PackGeo{P.pack, P.U, L}, (size_t)pc.rt * H + lane / L, P.n_out, P.n_in,
                       A.codes, A.exps, P.out_q32, P.out_f32, P.status);
        if (sh)
          checked_row<T>(PackGeo{P.pack2, P.U, L}, (size_t)pc.rt * H + lane / L, P.n_out,
                         P.n_in, A.codes, A.exps, P.out2_q32, P.out2_f32, P.status2);
      }
      done = lead;
    } else {
      for (int o = 1; o < L; o <<= 1) {  // the L lanes of a row combine
        const unsigned long long lo = __shfl_xor_sync(0xFFFFFFFFu, acc.lo, o);
        const unsigned long long hi = __shfl_xor_sync(0xFFFFFFFFu, acc.hi, o);
        acc_add(acc, lo, hi);
        if (sh) {
          const unsigned long long lo2 = __shfl_xor_sync(0xFFFFFFFFu, acc2.lo, o);
          const unsigned long long hi2 = __shfl_xor_sync(0xFFFFFFFFu, acc2.hi, o);
          acc_add(acc2, lo2, hi2);
        }
      }
      bool fin = P.npieces == 1;
      if (!fin) {
        Acc128 *dst = P.part + (((size_t)pc.rt * P.npieces + pc.q) << sh) * 32 + lane;
        dst->lo = acc.lo;
        dst->hi = acc.hi;
        if (sh) {
          dst[32].lo = acc2.lo;
          dst[32].hi = acc2.hi;
        }
        __syncwarp();
        fence_acq_rel_gpu();
        unsigned ticket = 0;
        if (lane == 0) ticket = atomicAdd(P.cnt + pc.rt, 1u);
        ticket = __shfl_sync(0xFFFFFFFFu, ticket, 0);
        fin = ticket == (unsigned)P.npieces - 1;
        if (fin) {
          fence_acq_rel_gpu();
          __syncwarp();
          acc_zero(acc);
          acc_zero(acc2);
          for (int qq = 0; qq < P.npieces; qq++) {
            const Acc128 *src = P.part + (((size_t)pc.rt * P.npieces + qq) << sh) * 32 + lane;
            acc_add(acc, __ldcg(&src->lo), __ldcg(&src->hi));
            if (sh) acc_add(acc2, __ldcg(&src[32].lo), __ldcg(&src[32].hi));
          }
          if (lane == 0) P.cnt[pc.rt] = 0u;  // ready for the next launch
        }
      }
      if (fin && slot == 0) {
        finish_row(acc, (size_t)pc.rt * H + lane / L, P.n_out, P.out_q32, P.out_f32, P.status,
                   PeerRows{});
        if (sh)
          finish_row(acc2, (size_t)pc.rt * H + lane / L, P.n_out, P.out2_q32, P.out2_f32,
                     P.status2, PeerRows{});
      }
      done = fin;
    }
    // -- the FFN hand-off: a 32-row block of h covers L row tiles of gate and of up; the last
    // of them to finish runs the block's SwiGLU --
    if (done && P.ffn >= 0 && sh && L == 1) {
      // this warp finished the block's gate and up rows itself (lane = row): the SwiGLU reads
      // back its own lanes' stores, so no counter and no fence stand between
      __syncwarp();
      ffn_block(g, P.ffn, pc.rt, lane);
    } else if (done && P.ffn >= 0) {
      // the block's row tiles count in: each of gate and of up, or each paired one
      const int blk = pc.rt / L;
      const int need = (2 >> sh) * (min(P.n_rt, (blk + 1) * L) - blk * L);
      __syncwarp();
      fence_acq_rel_gpu();
      unsigned old = 0;
      if (lane == 0) old = atomicAdd(g.ffn[P.ffn].pair + blk, 1u);
      old = __shfl_sync(0xFFFFFFFFu, old, 0);
      if (old == (unsigned)need - 1) {
        if (lane == 0) g.ffn[P.ffn].pair[blk] = 0u;  // ready for the next launch
        fence_acq_rel_gpu();
        __syncwarp();
        ffn_block(g, P.ffn, blk, lane);
      }
    }
    if (!copies_ok) break;  // the ring's phases are lost: this warp stops
    if (xn >= 0) us.advance(pn);
    x = xn;
    pc = pn;
    act_pre = next_pre;
  }

  // no copy may land in this CTA's shared memory after it exits
  while (us.k_fold < us.k_issue) {
    uint8_t *sl;
    us.wait_front(sl);
    us.k_fold++;
  }
  // the last CTA out resets the launch's counters and flags
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    if (atomicAdd(&g.ctl->exit, 1u) == gridDim.x - 1) {
      g.ctl->queue = 0u;
      g.ctl->abort = 0u;
      for (int f = 0; f < g.n_ffn; f++) {
        g.ctl->ready[f] = 0u;
        g.ctl->flag[f] = 0u;
        for (int k = 0; k < 4; k++) g.ctl->stats[f][k] = 0;
      }
      __threadfence();
      g.ctl->exit = 0u;
    }
  }
}

}  // namespace


// ---- host ---------------------------------------------------------------------------------------

struct PlanHost {
  uint32_t type = 0;
  int n_proj = 0, n_ffn = 0, total = 0;
  unsigned grid = 0;
  int block = 0;
  size_t smem = 0;
  void *dev = nullptr;  // records, control block and scratch in one allocation
  PlanProjD *proj = nullptr;
  PlanActD *act = nullptr;
  PlanFfnD *ffn = nullptr;
  PlanCtl *ctl = nullptr;
};

namespace {

size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

template <uint32_t T>
cudaError_t plan_geometry(int n_proj, int sm_count, unsigned &grid, int &block, size_t &smem) {
  block = PlanShape<T>::kThreads;
  smem = plan_fixed_smem<T>() + (((size_t)n_proj * 4 + 15) & ~(size_t)15);
  cudaError_t e = cudaFuncSetAttribute(plan_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, plan_kernel<T>, block, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  per_sm = std::min(per_sm, PlanShape<T>::kCtas);
  grid = (unsigned)(sm_count * per_sm);  // co-resident: every wait ends
  return cudaSuccess;
}

template <uint32_t T>
cudaError_t plan_launch(const PlanHost &h, const PlanArgs &a, cudaStream_t stream, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(h.grid);
  cfg.blockDim = dim3(h.block);
  cfg.dynamicSmemBytes = h.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, plan_kernel<T>, a);
}

// Records of one plan, checked: the FFNs' gate and up projections (index per FFN), and for every
// projection the FFN whose activation it reads (-1 for a resident one).
int plan_check(const PlanSpec &s, std::vector<int> &gate, std::vector<int> &up,
               std::vector<int> &reads) {
  const int n_proj = (int)s.projs.size(), n_act = (int)s.acts.size(), n_ffn = (int)s.ffns.size();
  if (n_proj < 1 || n_proj > kPlanMaxProj || n_ffn > kPlanMaxFfn) return APX_ERR_INVALID_ARGUMENT;
  const uint32_t type = s.projs[0].type;
  for (const PlanSpec::Act &x : s.acts)
    if (!x.codes || !x.exps || !x.desc || x.ffn < -1 || x.ffn >= n_ffn)
      return APX_ERR_INVALID_ARGUMENT;
  reads.assign(n_proj, -1);
  for (int i = 0; i < n_proj; i++) {
    const PlanSpec::Proj &p = s.projs[i];
    if (p.type != type || !p.pack || p.n_out == 0 || p.n_in == 0 || p.act < 0 ||
        p.act >= n_act || p.ffn < -1 || p.ffn >= n_ffn || !p.status || p.plan.L < 1 ||
        p.plan.units < 1)
      return APX_ERR_INVALID_ARGUMENT;
    reads[i] = s.acts[p.act].ffn;
  }
  gate.assign(n_ffn, -1);
  up.assign(n_ffn, -1);
  for (int i = 0; i < n_proj; i++) {
    const PlanSpec::Proj &p = s.projs[i];
    if (p.ffn < 0) continue;
    if (p.role != 0 && p.role != 1) return APX_ERR_INVALID_ARGUMENT;
    int &slot = p.role == 0 ? gate[p.ffn] : up[p.ffn];
    if (slot != -1) return APX_ERR_INVALID_ARGUMENT;
    slot = i;
  }
  for (int f = 0; f < n_ffn; f++) {
    const PlanSpec::Ffn &x = s.ffns[f];
    if (gate[f] < 0 || up[f] < 0 || x.out_act < 0 || x.out_act >= n_act ||
        s.acts[x.out_act].ffn != f || x.n_peers < 0 || x.n_peers > 7)
      return APX_ERR_INVALID_ARGUMENT;
    for (int p = 0; p < x.n_peers; p++)
      if (!x.peer_codes[p] || !x.peer_exps[p] || !x.peer_desc[p]) return APX_ERR_INVALID_ARGUMENT;
    const PlanSpec::Proj &pg = s.projs[gate[f]], &pu = s.projs[up[f]];
    if (pg.n_out != pu.n_out || pg.n_in != pu.n_in || pg.act != pu.act ||
        pg.plan.L != pu.plan.L || !pg.out_q32 || !pu.out_q32)
      return APX_ERR_INVALID_ARGUMENT;
    // readers of the FFN's activation come after both of its projections, at its width
    for (int i = 0; i < n_proj; i++)
      if (reads[i] == f && (i <= std::max(gate[f], up[f]) || s.projs[i].n_in != pg.n_out))
        return APX_ERR_INVALID_ARGUMENT;
  }
  return APX_OK;
}

}  // namespace

int plan_build(const PlanSpec &s, int sm_count, PlanHost **out) {
  *out = nullptr;
  std::vector<int> gate, up, reads;
  int rc = plan_check(s, gate, up, reads);
  if (rc != APX_OK) return rc;
  const int n_proj = (int)s.projs.size(), n_act = (int)s.acts.size(), n_ffn = (int)s.ffns.size();
  const uint32_t type = s.projs[0].type;
  unsigned grid = 0;
  int block = 0;
  size_t smem = 0;
  cudaError_t e;
  switch (type) {
    case kQ8_0: e = plan_geometry<kQ8_0>(n_proj, sm_count, grid, block, smem); break;
    case kQ4_K: e = plan_geometry<kQ4_K>(n_proj, sm_count, grid, block, smem); break;
    case kQ6_K: e = plan_geometry<kQ6_K>(n_proj, sm_count, grid, block, smem); break;
    default: return APX_ERR_INVALID_ARGUMENT;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return APX_ERR_CUDA;
  }
  const long long V = (long long)grid * (block / 32);

  // Every FFN's gate and up run as one paired record (the up's own record takes no pieces):
  // their units alternate over one staged activation, and the warp finishing a row tile runs
  // its SwiGLU block directly.  APX_PLAN_PAIR=0 keeps them apart (hand-off by counters).
  static const bool pair_on = [] {
    const char *v = std::getenv("APX_PLAN_PAIR");
    return !(v && v[0] == '0');
  }();
  std::vector<int> partner(n_proj, -1), dropped(n_proj, 0);
  if (pair_on)
    for (int f = 0; f < n_ffn; f++) {
      partner[gate[f]] = up[f];
      dropped[up[f]] = 1;
    }

  // Pieces: at most kPlanPiece units, fewer when the plan is short, so that every warp of the
  // grid gets about two.
  std::vector<int> n_rt(n_proj), npieces(n_proj), plen(n_proj);
  long long units = 0;
  for (int i = 0; i < n_proj; i++) {
    const PlanSpec::Proj &p = s.projs[i];
    const int H = 32 / p.plan.L;
    n_rt[i] = (int)((p.n_out + H - 1) / H);
    units += (long long)n_rt[i] * p.plan.units;
  }
  const int plen_t = (int)std::max<long long>(1, std::min<long long>(kPlanPiece, units / (2 * V)));
  long long total = 0;
  for (int i = 0; i < n_proj; i++) {
    const int U = s.projs[i].plan.units;
    if (dropped[i]) {  // streamed by its gate's record
      npieces[i] = 0;
      plen[i] = 1;
      continue;
    }
    const int Uv = partner[i] >= 0 ? 2 * U : U;  // units a row tile streams
    npieces[i] = (Uv + plen_t - 1) / plen_t;
    plen[i] = (U + npieces[i] - 1) / npieces[i];  // in real units: a pair stays in one piece
    npieces[i] = (U + plen[i] - 1) / plen[i];
    total += (long long)n_rt[i] * npieces[i];
  }
  if (total > INT_MAX / 2) return APX_ERR_TOO_LARGE;

  // Queue order by dependency level: a projection reading a resident activation has level 0,
  // one reading FFN f's activation the level of f's gate and up plus one.  Within a level the
  // FFN producers (gate / up) go first and the other projections after them, each group in the
  // given order: by the time a warp reaches a level's readers, every FFN they read had the whole
  // level's other work to finish in.
  std::vector<int> level(n_proj, 0), ffn_level(n_ffn, -1);
  for (int i = 0; i < n_proj; i++) {  // producers come before their readers (plan_check)
    level[i] = reads[i] < 0 ? 0 : ffn_level[reads[i]] + 1;
    const int f = s.projs[i].ffn;
    if (f >= 0) ffn_level[f] = std::max(ffn_level[f], level[i]);
  }
  std::vector<int> order(n_proj);
  for (int i = 0; i < n_proj; i++) order[i] = i;
  std::stable_sort(order.begin(), order.end(), [&](int a0, int b0) {
    const int ka = 2 * level[a0] + (s.projs[a0].ffn >= 0 ? 0 : 1);
    const int kb = 2 * level[b0] + (s.projs[b0].ffn >= 0 ? 0 : 1);
    return ka < kb;
  });

  // device records, in queue order
  std::vector<PlanProjD> pd(n_proj);
  std::vector<size_t> part_off(n_proj, 0), cnt_off(n_proj, 0), pair_off(n_ffn, 0);
  size_t scratch = 0;
  long long first = 0;
  for (int q = 0; q < n_proj; q++) {
    const int i = order[q];
    const PlanSpec::Proj &p = s.projs[i];
    PlanProjD &d = pd[q];
    d = PlanProjD{};
    d.pack = p.pack;
    d.out_q32 = p.out_q32;
    d.out_f32 = p.out_f32;
    d.status = p.status;
    d.n_out = p.n_out;
    d.n_in = p.n_in;
    d.L = p.plan.L;
    d.U = p.plan.units;
    d.n_rt = n_rt[i];
    d.npieces = npieces[i];
    d.plen = plen[i];
    d.piece0 = (int)first;
    d.act = p.act;
    d.ffn = p.ffn;
    if (partner[i] >= 0) {
      const PlanSpec::Proj &u = s.projs[partner[i]];
      d.paired = 1;
      d.pack2 = u.pack;
      d.out2_q32 = u.out_q32;
      d.out2_f32 = u.out_f32;
      d.status2 = u.status;
    }
    first += (long long)n_rt[i] * npieces[i];
    if (d.npieces > 1) {
      part_off[q] = scratch;
      scratch += al256((size_t)d.n_rt * d.npieces * (1 + d.paired) * 32 * sizeof(Acc128));
      cnt_off[q] = scratch;
      scratch += al256((size_t)d.n_rt * 4);
    }
  }
  std::vector<PlanActD> ad(n_act);
  for (int a = 0; a < n_act; a++) {
    const PlanSpec::Act &x = s.acts[a];
    ad[a] = PlanActD{x.codes, x.exps, static_cast<const ActDesc *>(x.desc), x.ffn, 0};
  }
  std::vector<PlanFfnD> fd(n_ffn);
  for (int f = 0; f < n_ffn; f++) {
    const PlanSpec::Ffn &x = s.ffns[f];
    const PlanSpec::Proj &pg = s.projs[gate[f]], &pu = s.projs[up[f]];
    PlanFfnD &d = fd[f];
    d = PlanFfnD{};
    d.gate = pg.out_q32;
    d.up = pu.out_q32;
    d.gate_status = pg.status;
    d.up_status = pu.status;
    d.h = x.h;
    d.codes = const_cast<int8_t *>(s.acts[x.out_act].codes);
    d.exps = const_cast<uint8_t *>(s.acts[x.out_act].exps);
    d.desc = static_cast<ActDesc *>(const_cast<void *>(s.acts[x.out_act].desc));
    d.status = x.status;
    d.n = pg.n_out;
    d.n_rt = (int)((pg.n_out + 31) / 32);
    d.carrier = x.carrier;
    d.refused = x.refused ? 1 : 0;
    d.n_peers = x.n_peers;
    for (int p = 0; p < x.n_peers; p++) {
      d.peer_codes[p] = x.peer_codes[p];
      d.peer_exps[p] = x.peer_exps[p];
      d.peer_desc[p] = static_cast<ActDesc *>(x.peer_desc[p]);
    }
    pair_off[f] = scratch;
    scratch += al256((size_t)d.n_rt * 4);
  }

  auto *h = new (std::nothrow) PlanHost;
  if (!h) return APX_ERR_OUT_OF_MEMORY;
  h->type = type;
  h->n_proj = n_proj;
  h->n_ffn = n_ffn;
  h->total = (int)total;
  h->grid = grid;
  h->block = block;
  h->smem = smem;
  const size_t o_proj = 0, o_act = al256(n_proj * sizeof(PlanProjD));
  const size_t o_ffn = o_act + al256(std::max(n_act, 1) * sizeof(PlanActD));
  const size_t o_ctl = o_ffn + al256(std::max(n_ffn, 1) * sizeof(PlanFfnD));
  const size_t o_scr = o_ctl + al256(sizeof(PlanCtl));
  const size_t bytes = o_scr + scratch;
  if (cudaMalloc(&h->dev, bytes) != cudaSuccess) {
    cudaGetLastError();
    delete h;
    return APX_ERR_OUT_OF_MEMORY;
  }
  uint8_t *base = static_cast<uint8_t *>(h->dev);
  for (int q = 0; q < n_proj; q++)
    if (pd[q].npieces > 1) {
      pd[q].part = reinterpret_cast<Acc128 *>(base + o_scr + part_off[q]);
      pd[q].cnt = reinterpret_cast<unsigned *>(base + o_scr + cnt_off[q]);
    }
  for (int f = 0; f < n_ffn; f++)
    fd[f].pair = reinterpret_cast<unsigned *>(base + o_scr + pair_off[f]);
  h->proj = reinterpret_cast<PlanProjD *>(base + o_proj);
  h->act = reinterpret_cast<PlanActD *>(base + o_act);
  h->ffn = reinterpret_cast<PlanFfnD *>(base + o_ffn);
  h->ctl = reinterpret_cast<PlanCtl *>(base + o_ctl);
  e = cudaMemset(h->dev, 0, bytes);
  if (e == cudaSuccess)
    e = cudaMemcpy(h->proj, pd.data(), n_proj * sizeof(PlanProjD), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && n_act)
    e = cudaMemcpy(h->act, ad.data(), n_act * sizeof(PlanActD), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && n_ffn)
    e = cudaMemcpy(h->ffn, fd.data(), n_ffn * sizeof(PlanFfnD), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaGetLastError();
    plan_free(h);
    return APX_ERR_CUDA;
  }
  *out = h;
  return APX_OK;
}

cudaError_t plan_run(const PlanHost &h, cudaStream_t stream, bool pdl) {
  PlanArgs a;
  a.proj = h.proj;
  a.act = h.act;
  a.ffn = h.ffn;
  a.ctl = h.ctl;
  a.n_proj = h.n_proj;
  a.n_ffn = h.n_ffn;
  a.total = h.total;
  a.V = (int)h.grid * (h.block / 32);
  switch (h.type) {
    case kQ8_0: return plan_launch<kQ8_0>(h, a, stream, pdl);
    case kQ4_K: return plan_launch<kQ4_K>(h, a, stream, pdl);
    case kQ6_K: return plan_launch<kQ6_K>(h, a, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

void plan_free(PlanHost *h) {
  if (!h) return;
  if (h->dev) cudaFree(h->dev);
  delete h;
}

}  // namespace apx
