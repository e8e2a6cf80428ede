// The chip decode on B200 (sm_100a): one thread-block cluster per machine (stream), the whole
// token loop inside one launch, the next token chosen and embedded on the device.
//
// What it computes is the reference's stock decode step (lx/lx/hf.py:169-184), as its
// megakernel does (lx/csrc/mega.cu:653-862): per token, every chip layer's Gated DeltaNet step
// and SwiGLU over their nonzero parts, then the output head's argmax. The arithmetic follows the
// CPU restatement in oracle/oracle.c operation for operation (the same lxb_math.h functions, the
// same fixed reduction orders), so the two agree bit for bit.
//
// How it maps to the hardware (the reference instead runs one 132-CTA persistent grid with a
// global-memory barrier per phase and fp32 atomics into a global accumulator):
//   - A cluster of C CTAs (C = 8 or 16, one per SM) runs one stream. Every CTA keeps a replica of
//     the residual row in shared memory. Cluster barriers (barrier.cluster, in hardware) separate
//     the steps; data crosses CTAs only through distributed shared memory (DSMEM).
//   - Residual rows are owned in contiguous blocks of 2560 / C. The owner computes every sum that
//     lands in its rows (down_proj and out_proj rows, sequentially in CSR order), re-evaluating
//     the few MLP units it needs itself, so no sum is split across CTAs and no atomic is used:
//     the results do not depend on timing. After a barrier every CTA pulls the C blocks back
//     into its replica with 16-byte DSMEM loads.
//   - One step per layer: the layer's GDN items (one live key head each) and its MLP (assuming
//     the GDN leaves the residual as it is) run side by side; if any item did write, an
//     out_proj step and the MLP again follow (two more barriers). The reference pairs only the
//     layers it measured (PAIR_LAYERS, lx/lx/mega.py:97); here every layer is paired.
//   - Value channels are kept lazily: their projections only matter on the steps a key of
//     their head fires (the delta rule's v) and for the conv windows the launch leaves behind.
//     Each step stores its GDN input row in a 4-step ring (device scratch); a firing key's
//     head recomputes its value channels' last four projections from it, and at the launch's
//     end every lazy window is rebuilt the same way. The reference evaluates every channel on
//     every step (lx/csrc/mega.cu:318-336); the results are the same bits.
//   - Independent streams are independent clusters: no inter-cluster communication at all.
// No device-wide barrier exists, so nothing spins on global memory; the only waits are
// hardware cluster barriers, which every CTA of a cluster reaches on the same cluster-uniform
// control path.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <climits>
#include <algorithm>
#include <atomic>
#include <mutex>
#include <new>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "../../include/lxb.h"
#include "lxb_math.h"
#include "lxb_plan.h"

namespace cg = cooperative_groups;

#define NT 512
#define H LXB_H
#define KD LXB_KD
#define VD LXB_VD
#define R LXB_R
#define BLKMAX (LXB_H / LXB_MINC)
#define LXB_MAXLAYERS 64
#define LXB_MAXPROD 4096
#define LXB_LOGMAX 512  // group steps: window shifts a CTA may undo (entries of 12 bytes)
#define LXB_NOLOG 0xffffffffu  // an undo log entry that undoes nothing
#define LXB_QLAYERS 32  // layers one quiet pass covers
#define LXB_QTASKS (LXB_QLAYERS * LXB_ITEMSLOTS)
#define LXB_QNONE 0xffffffffu
#define LXB_QFULL 0x40000000u
#define LXB_LONGROWS 64  // out_proj / down_proj rows of a CTA summed by a warp each (the rest by
#define LXB_LONG 32      // a thread each): rows with more than LXB_LONG entries
#define LXB_QOUT 0x80000000u   // (qinfo) the item's head has out_proj entries
#ifndef LXB_GROUPS
#define LXB_GROUPS 1    // runs of GDN-only layers as optimistic group steps
#endif

struct Dev {
  const lxb_layer* layers;
  const lxb_item* items;
  const lxb_chan* chans;
  const uint32_t* ent;
  const lxb_unit* units;
  const lxb_owner* owners;
  const int32_t* i32;
  const uint16_t* u16;
  const lxb_headcta* headcta;
  const uint64_t* hcodes;
  int n_layers, C, blk, n_vocab, n_dense, final_norm;
  float eps;
  int64_t n_embed_rows;
  int offset;
  float htab[4];
  int dense_cols[LXB_MAXDENSE];
  const uint32_t* hsp;  // the head columns with sparse entries, a bitmask (null: none)
  uint32_t* status;  // [0] bits, [1] first stream, [2] first step
  const unsigned char* blobs;  // the step blobs
  const lxb_blobref* blobidx;  // [(n_layers + 1) * C]
  const int32_t* winmap;       // (layer, conv channel) pairs
  const int32_t* winidx;       // per CTA: (offset, count) into winmap
  int nbuf;                    // staging buffers in shared memory (1 or 2)
  int stage;                   // bytes per staging buffer: larger blobs are read where they are
};

struct Run {
  const uint64_t* state_ptrs;  // [stream][layer][2]
  uint32_t* bitmaps;           // [stream][layer][128][8]
  uint16_t* ring;              // [stream][layer][4][2560]: the GDN input rows of the last 4 steps
  float* ring_r;               // [stream][layer][4]: their RMSNorm factors
  const uint16_t* embed;
  const int32_t* forced;
  int n_forced, n_tokens;
  int32_t* preds;
  int32_t* inputs;
  unsigned long long* prof;  // optional: [stream][cta][LXB_PROF_N] cycle counters, accumulated
  int n_streams;               // decoding clusters; the clusters after them are head helpers
  int n_help;                  // head helper clusters (a single stream only), slices 1..n_help
  float* hx;                   // [2560]: the head's input, published by the decoding cluster
  unsigned long long* hseq;    // the token whose head input hx holds (epoch | token + 1)
  uint4* hpart;                // [slice * cluster + rank]: a helper's maximum {v, row, seq lo, hi}
  unsigned long long epoch;    // this launch's tag (launch count << 32): stale words never match
  int help_drill;              // the helpers start but never answer (the fallback's test)
  lxb_typing typing;           // the device typing queue (keys == null: off)
};

// profile sections (lxb_plan_set_profile): cycles spent per CTA
enum {
  PR_NORM,     // sum of squares, norms, ring write
  PR_ITEMS,    // GDN items
  PR_MLP,      // MLP owner (the paired step)
  PR_SYNC,     // the paired step's cluster barrier
  PR_PULL,     // pulling the residual after a step
  PR_FIXUP,    // a write's out_proj step and MLP redo, barriers included
  PR_HEAD,     // the head: norm, rows, barrier, reduce
  PR_EMBED,    // the next token's embedding
  PR_FIXUPS,   // count: fix-up steps
  PR_TOKENS,   // count: tokens
  PR_WAIT,     // waiting for a staged blob
  PR_POLLS,    // count: staging polls that found the copy still in flight
  PR_TAKESYNC, // the block barrier after the staging wait
  PR_BARRIERS, // count: cluster barriers in the token loop
  PR_GITEMS,   // group steps: quiet pass and items
  PR_GSYNC,    // group steps: the cluster barrier
  PR_GFIXUP,   // group steps: undo, out_proj fix-ups
  PR_FXMLP,    // a paired step's fix-up: the MLP again, its barrier
  PR_FXOUT,    // a paired step's fix-up: the out_proj rows (before their push and barrier)
  PR_N
};

struct __align__(16) Smem {
  alignas(16) float x[H];          // the residual replica (bf16 values)
  float xn[H];                     // input_layernorm(x) (bf16 values)
  float xm[H];                     // post_attention_layernorm(x) or the final norm
  alignas(16) float own[2][BLKMAX];  // this CTA's rows after the step, by step parity
  alignas(16) uint16_t xin[2][H];  // the residual as the owners push it (bf16), by step parity
  float buf[LXB_NSLOT];            // an item's q | k | v
  float qval[KD], kval[KD];        // nonzero l2-normed query (x 1/16) and key values
  int qidx[KD], kidx[KD];
  float ob[R][VD];                 // o per value head (bf16 values)
  float beta[R], g[R];
  uint32_t dbm[R][8];              // a decaying item's nonzero-row bitmaps
  uint32_t nzm[R][8];              // ... the rows still nonzero after this token's decay
  float ge[R];                     // ... exp(g) per value head (1: no decay now)
  int drows;                       // ... the rows their bitmaps hold (decaying heads)
  float red[40];
  int nq, nk;
  int qkn;                         // the q / k lists are l2-normed already (eager_block)
  uint32_t vhmask[LXB_ITEMSLOTS];  // value heads with output, per item slot
  int vhlay[LXB_ITEMSLOTS];        // the layer and token whose item last set the slot's vhmask
  int vhtok[LXB_ITEMSLOTS];
  int gkey[2];                     // group steps, by parity: 2 layer + (0 pending | 1 wrote)
  uint32_t lmeta[LXB_LOGMAX];      // undo log: window index | item << 10 | (layer - lo) << 12
  uint2 lold[LXB_LOGMAX];          // the window before the shift
  uint32_t qinfo[LXB_MAXLAYERS][LXB_ITEMSLOTS];  // this CTA's items per layer (blob order):
                                   // first channel | n_eager << 24 if a quiet pass may take it,
                                   // LXB_QFULL if not, LXB_QNONE past the last
  uint4 qtask[LXB_QTASKS];         // a quiet pass's items: k | layer << 8, log, channel, qinfo
  int qfull[LXB_QLAYERS];          // per layer of the pass: the items that need a full run
  int qn, qlog, qnch;              // the pass's item count, undo log entries, channels
  uint32_t qbad;                   // an MLP step's items with a nonzero key (or query) output
  int wflag[2];                    // some item of the step wrote (pushed by the writer)
  int kmask[LXB_NK];               // out_proj step: active value heads per key head
  int lrows[LXB_LONGROWS];         // owned rows with many entries, summed by a warp each
  int nlong;
  unsigned long long bigm;         // layers whose every item is too big for a group step's
                                   // speculation (many query/key channels, windows in global
                                   // memory, or a decay): they run as steps of their own
  unsigned long long pcs[PR_N];    // the profile's counters (thread 0's timeline)
  unsigned long long upm;          // layers whose GDN wrote at the last token: their MLP waits
                                   // for the out_proj rows instead of running beside the items
  uint32_t kinfo[LXB_MAXLAYERS][LXB_NK];  // per layer and key head: its item's slot | cta << 8 |
                                   // 1 << 16 (0: no item), for the out_proj step's gather
  alignas(16) uint16_t on[LXB_ITEMSLOTS][R * VD];  // the gated norm's output per item slot
  union {
    alignas(16) uint16_t onall[LXB_NK][R * VD];  // gathered for the out_proj step
    struct {
      float xr[H];                 // input_layernorm of an earlier step's residual
      uint16_t pw[4][LXB_NSLOT];   // lazy channels: their projections at 4 steps
    } lz;
    struct {
      alignas(16) uint16_t xb[3][H];  // a key's firing: the 3 earlier steps' input norms
    } lf;
    float htg[LXB_MAXDENSE / 4][256];  // head: per group of 4 dense columns, each code's sum
  };  // (each member lives within one step: an item, an out_proj step or the head)
  float hbuf[LXB_MAXUNITS];        // MLP unit outputs
  float prod[LXB_MAXPROD];         // MLP gate/up products, in the units' entry order
  float bestv;
  int besti;
  int tok;
  int broken;                      // a staging wait gave up: blobs are not used any more
  alignas(8) unsigned long long mbar[2];  // staging buffers' transaction barriers
  const unsigned char* bsrc[2];     // the blob each buffer's phase stands for: the buffer, or the
                                    // blob in global memory when it is larger than a buffer
  uint32_t hspm[H / 32];            // the head columns with sparse entries
  lxb_layer layers[LXB_MAXLAYERS];  // the layer descriptors
  uint64_t sptr[LXB_MAXLAYERS][2];  // this stream's state pointers per layer
  lxb_blobref bref[LXB_MAXLAYERS + 1];  // this CTA's step blobs (the head's last)
  alignas(8) uint2 win[LXB_MAXWIN];  // resident query/key conv windows
  int nwin, win0;                   // their count and offset in the window map
  int help_dead;                    // the helpers stopped answering: the cluster does every slice
  float cv, hv, gv;                 // the cluster's first maximum; with the helpers'; rank 0's
  int ci, hi, gi, hok;              // gathering; their rows; whether every helper answered
  int tq_k, tq_wait, tq_left;       // typing: keys typed, the RX FIFO's count, keys left in a batch
};

// --- block reductions in the canonical orders -------------------------------------------------
__device__ __forceinline__ float warp_xor_sum(float s) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s = lx_add(s, __shfl_xor_sync(0xffffffffu, s, off));
  return s;
}

// lane t sums x[t + 512 i]^2 (i = 0..4), butterfly per warp, butterfly over the 16 warp sums
__device__ float block_ssq(Smem& sm, const float* x) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float s = lx_mul(x[t], x[t]);
#pragma unroll
  for (int i = 1; i < 5; i++) s = lx_add(s, lx_mul(x[t + 512 * i], x[t + 512 * i]));
  s = warp_xor_sum(s);
  if (lane == 0) sm.red[warp] = s;
  __syncthreads();
  // every warp reduces the 16 warp sums itself (the same butterfly, so the same bits
  // everywhere); every caller passes another block barrier before the next call writes red
  float v = lane < 16 ? sm.red[lane] : 0.0f;
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) v = lx_add(v, __shfl_xor_sync(0xffffffffu, v, off));
  const float r = __shfl_sync(0xffffffffu, v, 0);
  return r;
}

__device__ __forceinline__ float norm_factor(const Dev& P, float ss) {
  return lx_rsqrt(lx_add(lx_div(ss, (float)H), P.eps));
}

// Qwen3_5RMSNorm with the factor r: out[c] = bf16(x[c] * r * (1 + w[c])), w the bf16 weight
// (a staged copy in shared memory)
__device__ void norm_into(float* out, const float* x, const uint16_t* w, float r) {
  for (int c = threadIdx.x; c < H; c += NT)
    out[c] = lx_rbf(lx_mul(lx_mul(x[c], r), lx_add(1.0f, lx_f(w[c]))));
}

// --- staging: bulk copies (TMA) of the next step's blob into shared memory --------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void stage_issue(const Dev& P, Smem& sm, unsigned char* stage, int buf,
                                            int L) {
  const lxb_blobref br = sm.bref[L];
  unsigned char* dst = stage + (size_t)buf * P.stage;
  const unsigned char* src = P.blobs + br.off;
  const uint32_t mb = smem_u32(&sm.mbar[buf]);
  // a blob larger than a buffer is read in global memory: the phase completes on the arrival
  // alone (no bytes expected), and the takers read the pointer published before it
  const bool staged = br.bytes <= P.stage;
  sm.bsrc[buf] = staged ? dst : src;
  // the buffer was last read through the generic proxy, by threads that have passed a block
  // barrier since: an async-proxy write after generic reads needs no proxy fence (the ordering
  // of the usual bulk-copy producer/consumer pipelines)
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mb),
               "r"(staged ? (uint32_t)br.bytes : 0u)
               : "memory");
  for (int o = 0; staged && o < br.bytes; o += 32768) {
    const uint32_t n = (uint32_t)min(32768, br.bytes - o);
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst + o)), "l"(src + o), "r"(n), "r"(mb)
        : "memory");
  }
}

// wait for a staging buffer (bounded by the global timer: a copy that never lands sets the
// status and stops every later use of the staged blobs instead of spinning forever)
__device__ __forceinline__ bool stage_wait(const Dev& P, Smem& sm, int buf, uint32_t phase,
                                           int s, int step, unsigned long long& polls) {
  const uint32_t mb = smem_u32(&sm.mbar[buf]);
  long long t0 = 0;
  for (int it = 0;; it++) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(mb), "r"(phase)
        : "memory");
    if (ok) return true;
    polls++;
    if (it == 0) t0 = clock64();
    if (clock64() - t0 > 4000000000ll) {  // ~2 s at the B200's clock
      if (threadIdx.x == 0) {
        if (atomicOr(P.status, LXB_S_STAGE) == 0) {
          P.status[1] = (uint32_t)s;
          P.status[2] = (uint32_t)step;
        }
      }
      return false;
    }
  }
}

// sequential dot over entries [e0, e0 + n) (column | bf16 << 16), loads issued 8 at a time
__device__ __forceinline__ float dotb(const uint32_t* __restrict__ ent, uint32_t e0, int n,
                                      const float* x) {
  float s = 0.0f;
  for (int e = 0; e < n; e += 8) {
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; k++) w[k] = e + k < n ? __ldg(ent + e0 + e + k) : 0u;
#pragma unroll
    for (int k = 0; k < 8; k++)
      if (e + k < n) s = lx_add(s, lx_mul(x[w[k] & 0xffffu], lx_f((uint16_t)(w[k] >> 16))));
  }
  return s;
}

// two sequential dots with their loads interleaved (a unit's gate and up rows)
__device__ __forceinline__ void dot2b(const uint32_t* __restrict__ ent, uint32_t ga, int gn,
                                      uint32_t ua, int un, const float* x, float& sg,
                                      float& su) {
  float a = 0.0f, b = 0.0f;
  const int m = gn > un ? gn : un;
  for (int e = 0; e < m; e += 8) {
    uint32_t wg[8], wu[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
      wg[k] = e + k < gn ? __ldg(ent + ga + e + k) : 0u;
      wu[k] = e + k < un ? __ldg(ent + ua + e + k) : 0u;
    }
#pragma unroll
    for (int k = 0; k < 8; k++)
      if (e + k < gn) a = lx_add(a, lx_mul(x[wg[k] & 0xffffu], lx_f((uint16_t)(wg[k] >> 16))));
#pragma unroll
    for (int k = 0; k < 8; k++)
      if (e + k < un) b = lx_add(b, lx_mul(x[wu[k] & 0xffffu], lx_f((uint16_t)(wu[k] >> 16))));
  }
  sg = a;
  su = b;
}

__device__ __forceinline__ void set_status(const Dev& P, uint32_t bit, int stream, int step) {
  if (atomicOr(P.status, bit) == 0) {
    P.status[1] = (uint32_t)stream;
    P.status[2] = (uint32_t)step;
  }
}

// sm.lz.xr = input_layernorm of step tau's residual at layer L, from the ring
__device__ void build_xr(const Dev& P, const Run& run, Smem& sm, int s, int L, int tau,
                         const uint16_t* w) {
  const size_t slot = ((size_t)s * P.n_layers + L) * 4 + (tau & 3);
  const uint4* xs = reinterpret_cast<const uint4*>(run.ring + slot * H);
  const float r = __ldcg(run.ring_r + slot);
  for (int k = threadIdx.x; k < H / 8; k += NT) {
    const uint4 v = __ldcg(xs + k);
    const uint32_t xw[4] = {v.x, v.y, v.z, v.w};
    const uint16_t* wv = w + 8 * k;
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const float xv = lx_f((uint16_t)(q & 1 ? xw[q >> 1] >> 16 : xw[q >> 1] & 0xffffu));
      sm.lz.xr[8 * k + q] = lx_rbf(lx_mul(lx_mul(xv, r), lx_add(1.0f, lx_f(wv[q]))));
    }
  }
  __syncthreads();
}

// Lazily kept channels [c0, c1) of an item: their projections P at the steps tau = base + p
// (p = 0..3) into sm.lz.pw[p][c - c0]. P of a step before the launch comes from the channel's conv
// window as the launch found it (a lazy channel's window is not written until the launch ends).
// `cur` is the current step (its input norm is sm.xn already), or a value no step has.
// taps_only: compute P only where the channel's tap p is nonzero (0 elsewhere: a zero tap's
// product is a signed zero, which leaves the conv sum as it is).
__device__ void lazy_proj(const Dev& P, const Run& run, Smem& sm, const lxb_item& it,
                          const uint16_t* conv, int s, int L, int base, int cur, bool taps_only,
                          int c0, int c1, const uint16_t* w) {
  const int t = threadIdx.x;
  for (int p = 0; p < 4; p++) {
    const int tau = base + p;
    const float* xsrc = nullptr;
    if (tau == cur) {
      xsrc = sm.xn;
    } else if (tau >= 0) {
      build_xr(P, run, sm, s, L, tau, w);
      xsrc = sm.lz.xr;
    }
    for (int c = c0 + t; c < c1; c += NT) {
      const lxb_chan* cp = P.chans + it.ch0 + c;
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(cp));
      uint16_t v = 0;
      if (taps_only && !((__ldg(reinterpret_cast<const uint4*>(cp) + 1).y >> p) & 1)) {
        v = 0;
      } else if (xsrc) {
        v = lx_rb(dotb(P.ent, a.x, (int)(a.y & 0xffffu), xsrc));
      } else {  // before the launch: the window holds P of steps -4..-1 at positions 0..3
        const uint2 win = *reinterpret_cast<const uint2*>(conv + (size_t)a.z * 4);
        const int pos = tau + 4;
        const uint32_t wd = pos < 2 ? win.x : win.y;
        v = (uint16_t)((pos & 1) ? wd >> 16 : wd & 0xffffu);
      }
      sm.lz.pw[p][c - c0] = v;
    }
    __syncthreads();
  }
}

__device__ __forceinline__ float d_silu(float x) { return lx_silu(x); }

// A key fired: the conv outputs at this step of the item's value channels with a nonzero tap,
// into sm.buf at their slots. The stock step's window would hold the channel's projections P at
// the last four steps: P(step) from sm.xn (this step's input norm, built by the caller), P at the
// three steps before from the residual ring (their input norms rebuilt once for all channels, as
// bf16, only for the tap positions some channel has), or, for steps before the launch, from the
// window as the launch found it. Every channel evaluates only its nonzero taps, all from one pass
// over its entries (each tap's dot still sequential from +0 in entry order).
__device__ void lazy_fire(const Dev& P, const Run& run, Smem& sm, const lxb_item& it,
                          const uint16_t* conv, int s, int L, int step, const uint16_t* w) {
  const int t = threadIdx.x;
  int need = 0;
  for (int p = 0; p < 3; p++)
    if (((it.tapu >> p) & 1) && step - 3 + p >= 0) need |= 1 << p;
  if (need) {
    for (int k = t; k < 3 * (H / 8); k += NT) {
      const int p = k / (H / 8), kk = k - p * (H / 8);
      if (!((need >> p) & 1)) continue;
      const size_t slot = ((size_t)s * P.n_layers + L) * 4 + ((step - 3 + p) & 3);
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(run.ring + slot * H) + kk);
      const float r = __ldcg(run.ring_r + slot);
      const uint32_t xw[4] = {v.x, v.y, v.z, v.w};
      const uint16_t* wv = w + 8 * kk;
      uint32_t o[4];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float x0 = lx_f((uint16_t)(xw[q] & 0xffffu)), x1 = lx_f((uint16_t)(xw[q] >> 16));
        const uint16_t y0 = lx_rb(lx_mul(lx_mul(x0, r), lx_add(1.0f, lx_f(wv[2 * q]))));
        const uint16_t y1 = lx_rb(lx_mul(lx_mul(x1, r), lx_add(1.0f, lx_f(wv[2 * q + 1]))));
        o[q] = (uint32_t)y0 | ((uint32_t)y1 << 16);
      }
      reinterpret_cast<uint4*>(sm.lf.xb[p])[kk] = make_uint4(o[0], o[1], o[2], o[3]);
    }
    __syncthreads();
  }
  for (int c = it.n_eager + t; c < it.n_eager + it.n_vneed; c += NT) {
    const uint4* cp = reinterpret_cast<const uint4*>(P.chans + it.ch0 + c);
    const uint4 a = __ldg(cp);      // entries, count | slot << 16, conv channel, taps 0-1
    const uint4 b = __ldg(cp + 1);  // taps 2-3, tap mask
    const uint32_t tm = b.y;
    int dm = 0;  // the taps whose P is a dot product (a nonzero tap at a step of this launch)
    for (int p = 0; p < 4; p++)
      if (((tm >> p) & 1) && step - 3 + p >= 0) dm |= 1 << p;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int n = (int)(a.y & 0xffffu);
    for (int e = 0; e < n; e += 8) {
      uint32_t wv[8];
#pragma unroll
      for (int q = 0; q < 8; q++) wv[q] = e + q < n ? __ldg(P.ent + a.x + e + q) : 0u;
#pragma unroll
      for (int q = 0; q < 8; q++) {
        if (e + q >= n) continue;
        const uint32_t col = wv[q] & 0xffffu;
        const float wf = lx_f((uint16_t)(wv[q] >> 16));
        if (dm & 1) acc[0] = lx_add(acc[0], lx_mul(lx_f(sm.lf.xb[0][col]), wf));
        if (dm & 2) acc[1] = lx_add(acc[1], lx_mul(lx_f(sm.lf.xb[1][col]), wf));
        if (dm & 4) acc[2] = lx_add(acc[2], lx_mul(lx_f(sm.lf.xb[2][col]), wf));
        if (dm & 8) acc[3] = lx_add(acc[3], lx_mul(sm.xn[col], wf));
      }
    }
    uint2 win = make_uint2(0u, 0u);
    if (tm & ~dm & 15) win = *reinterpret_cast<const uint2*>(conv + (size_t)a.z * 4);
    const uint16_t taps[4] = {(uint16_t)(a.w & 0xffffu), (uint16_t)(a.w >> 16),
                              (uint16_t)(b.x & 0xffffu), (uint16_t)(b.x >> 16)};
    float y = 0.0f;
#pragma unroll
    for (int p = 0; p < 4; p++) {
      uint16_t pv = 0;
      if ((dm >> p) & 1) {
        pv = lx_rb(acc[p]);
      } else if ((tm >> p) & 1) {  // a step before the launch: positions 0..3 hold steps -4..-1
        const int pos = step + 1 + p;
        const uint32_t wd = pos < 2 ? win.x : win.y;
        pv = (uint16_t)((pos & 1) ? wd >> 16 : wd & 0xffffu);
      }
      y = lx_add(y, lx_mul(lx_f(taps[p]), lx_f(pv)));
    }
    const float yb = lx_rbf(y);
    sm.buf[a.y >> 16] = yb == 0.0f ? yb : lx_rbf(d_silu(yb));
  }
}

// --- a GDN item: one live key head of one layer --------------------------------------------------
// transformers' l2norm in bf16 over a compacted list (the nonzero entries in ascending order):
// x * rsqrt(sum(x * x) + 1e-6), the bf16 squares summed sequentially from +0 by one lane
__device__ __forceinline__ float l2_inv(const float* val, int n) {
  float sq = 0.0f;
  for (int i = 0; i < n; i++) sq = lx_add(sq, lx_rbf(lx_mul(val[i], val[i])));
  return lx_rbf(lx_rsqrt(lx_rbf(lx_add(lx_rbf(sq), 1e-6f))));
}

// input_layernorm(x)[c] for one column: bf16(x[c] * r * (1 + w[c])), as norm_into computes it
__device__ __forceinline__ float xn_at(const Smem& sm, const uint16_t* w, float r, uint32_t c) {
  return lx_rbf(lx_mul(lx_mul(sm.x[c], r), lx_add(1.0f, lx_f(w[c]))));
}

// A channel's conv step: the window (taps 0..2 of the last three projections) shifted with this
// step's projection Pv (nw), the conv output over it (taps t01, t23: bf16 pairs, low half first)
// in order from +0, and its silu in bf16 (0 stays 0)
__device__ __forceinline__ float conv_step(const uint2 win, uint16_t Pv, uint32_t t01, uint32_t t23,
                                           uint2& nw) {
  const uint16_t n0 = (uint16_t)(win.x >> 16), n1 = (uint16_t)(win.y & 0xffffu),
                 n2 = (uint16_t)(win.y >> 16);
  nw = make_uint2((uint32_t)n0 | ((uint32_t)n1 << 16), (uint32_t)n2 | ((uint32_t)Pv << 16));
  float y = 0.0f;
  y = lx_add(y, lx_mul(lx_f((uint16_t)(t01 & 0xffffu)), lx_f(n0)));
  y = lx_add(y, lx_mul(lx_f((uint16_t)(t01 >> 16)), lx_f(n1)));
  y = lx_add(y, lx_mul(lx_f((uint16_t)(t23 & 0xffffu)), lx_f(n2)));
  y = lx_add(y, lx_mul(lx_f((uint16_t)(t23 >> 16)), lx_f(Pv)));
  const float yb = lx_rbf(y);
  return yb == 0.0f ? yb : lx_rbf(d_silu(yb));
}

// One eager (query/key) channel: in_proj_qkv row over the staged entries (the input norm taken
// per column), conv window shift (resident in shared memory, or in global), conv output with
// silu in bf16. pr: the row's products, computed beforehand by the whole block (then only the
// sequential sum is this thread's), or null (the products here). zin: every product of the item
// is +0 or -0 (most steps: the residual is sparse), so the sequential sum from +0 is +0.
__device__ __forceinline__ float eager_channel(Smem& sm, const unsigned char* B, const uint4 a,
                                               const uint4 b, uint16_t* conv, const uint16_t* w,
                                               float r, const float* pr, bool zin) {
  const uint32_t* e = reinterpret_cast<const uint32_t*>(B + a.x);
  const int ne = (int)(a.y & 0xffffu);
  uint2* wp = b.y != LXB_NOWIN ? &sm.win[b.y] : reinterpret_cast<uint2*>(conv + (size_t)a.z * 4);
  const uint2 win = *wp;
  float ps = 0.0f;
  if (zin) {
  } else if (pr) {  // in batches of 8, the last one partial: every batch's loads in flight together
    for (int k = 0; k < ne; k += 8) {
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; q++) v[q] = k + q < ne ? pr[k + q] : 0.0f;
#pragma unroll
      for (int q = 0; q < 8; q++)
        if (k + q < ne) ps = lx_add(ps, v[q]);
    }
  } else {
    for (int k = 0; k < ne; k++)
      ps = lx_add(ps, lx_mul(xn_at(sm, w, r, e[k] & 0xffffu), lx_f((uint16_t)(e[k] >> 16))));
  }
  uint2 nw;
  const float v = conv_step(win, lx_rb(ps), a.w, b.x, nw);
  *wp = nw;
  return v;
}

// Pieces of an item: the rare paths (many query/key channels, decay, a key firing, output).

// a row dot over staged entries with the input norm taken per column (b / a rows, z rows)
__device__ __forceinline__ float xrow_dot(const Smem& sm, const uint32_t* e, int ne,
                                          const uint16_t* w_in, float r_in) {
  float d = 0.0f;
  for (int k = 0; k < ne; k++)
    d = lx_add(d, lx_mul(xn_at(sm, w_in, r_in, e[k] & 0xffffu), lx_f((uint16_t)(e[k] >> 16))));
  return d;
}

// many query/key channels: a dense q | k buffer, then compaction by warps 0 and 1
__device__ __forceinline__ void eager_block(Smem& sm, const unsigned char* B, const lxb_bitem& bi,
                                         uint16_t* conv, const uint16_t* w_in, float r_in,
                                         const float* pre_base, uint32_t e_first, bool zin) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const uint4* ch = reinterpret_cast<const uint4*>(B + bi.eager);
  for (int k = t; k < 2 * KD; k += NT) sm.buf[k] = 0.0f;
  __syncthreads();
  for (int c = t; c < bi.n_eager; c += NT) {
    const uint4 a = ch[2 * c], b = ch[2 * c + 1];
    sm.buf[a.y >> 16] = eager_channel(sm, B, a, b, conv, w_in, r_in,
                                      pre_base ? pre_base + (a.x - e_first) / 4u : nullptr, zin);
  }
  __syncthreads();
  if (warp < 2) {
    const float* xv = sm.buf + warp * KD;
    int* idx = warp ? sm.kidx : sm.qidx;
    float* val = warp ? sm.kval : sm.qval;
    int n = 0;
    for (int base = 0; base < KD; base += 32) {
      const float v = xv[base + lane];
      const unsigned m = __ballot_sync(0xffffffffu, v != 0.0f);
      if (v != 0.0f) {
        const int k = n + __popc(m & ((1u << lane) - 1u));
        idx[k] = base + lane;
        val[k] = v;
      }
      n += __popc(m);
    }
    __syncwarp();
    float inv = 0.0f;
    if (lane == 0 && n) inv = l2_inv(val, n);
    inv = __shfl_sync(0xffffffffu, inv, 0);
    for (int i = lane; i < n; i += 32) {
      const float vn = lx_rbf(lx_mul(val[i], inv));
      val[i] = warp ? vn : lx_mul(vn, 0.0625f);  // the query times 256^-0.5
    }
    if (lane == 0) (warp ? sm.nk : sm.nq) = n;
    if (t == 0) {
      sm.vhmask[bi.slot] = 0;
      sm.qkn = 1;
    }
  }
}

// g = -exp(A_log) * softplus(bf16(a . x) + dt_bias) of value head r, for a head that can decay
__device__ __forceinline__ float item_g(const Smem& sm, const unsigned char* B, const lxb_bitem& bi,
                                     int r, const uint16_t* w_in, float r_in) {
  const int32_t* brows = reinterpret_cast<const int32_t*>(B + bi.rows);
  const uint16_t* prm = reinterpret_cast<const uint16_t*>(B + bi.prm);
  const float d = xrow_dot(sm, reinterpret_cast<const uint32_t*>(B + brows[2 * (R + r)]),
                           brows[2 * (R + r) + 1], w_in, r_in);
  const float A = -lx_exp(lx_f(prm[r]));
  return lx_mul(A, lx_softplus(lx_add(lx_rbf(d), lx_f(prm[R + r]))));
}

// A key fired: beta = bf16(sigmoid(bf16(b . x))) (warp 1), and the value channels' conv outputs
// at this step into their q | k | v slots (the others zero). Ends with a block barrier.
__device__ __forceinline__ void item_fire(const Dev& P, const Run& run, Smem& sm,
                                       const unsigned char* B, const lxb_bitem& bi,
                                       uint16_t* conv, int s, int L, int step,
                                       const uint16_t* w_in, float r_in) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  if (warp == 1 && lane < R) {
    const int32_t* brows = reinterpret_cast<const int32_t*>(B + bi.rows);
    const float d = xrow_dot(sm, reinterpret_cast<const uint32_t*>(B + brows[2 * lane]),
                             brows[2 * lane + 1], w_in, r_in);
    sm.beta[lane] = lx_rbf(lx_sigmoid(lx_rbf(d)));
  }
  for (int k = t; k < R * VD; k += NT) sm.buf[2 * KD + k] = 0.0f;
  const lxb_item it = P.items[bi.item];
  if (it.n_vneed) {
    norm_into(sm.xn, sm.x, w_in, r_in);  // this step's input norm, for the lazy projections
    __syncthreads();
    lazy_fire(P, run, sm, it, conv, s, L, step, w_in);
  }
  __syncthreads();
}

// The decay of an item's value heads: every row that may be nonzero (the bitmaps, staged in
// sm.dbm) times exp(g) (sm.ge), over the whole block: thread (group grp = t / 128, column j)
// takes, for every decaying head, the rows r with r % 4 == grp, D rows' loads in flight per
// round, so a head whose rows all stay nonzero (a slow decay holds its values at small
// subnormals, which its factor rounds back to themselves) costs a quarter of what one thread
// group alone would. A row whose 128 columns all decayed to zero leaves the bitmap (sm.nzm; zero
// rows stay zero).
// A thread's two value heads rA and rA + 4 (SA, SB at row 0, its column): each head's rows
// gathered across its bitmap words, 12 loads in flight per round. The cheaper walk when the
// bitmaps hold few rows (the block's threads then have little to share out).
__device__ __forceinline__ void item_decay_pairs(Smem& sm, float* SA, float* SB, int rA) {
  const int lane = threadIdx.x & 31;
  constexpr int HPT = 2, D = 6, HS = 4;
  float* S[HPT] = {SA, SB};
  float e[HPT];
  int w[HPT];
  uint32_t m[HPT];
  bool on[HPT];
#pragma unroll
  for (int k = 0; k < HPT; k++) {
    e[k] = sm.ge[rA + k * HS];
    on[k] = e[k] != 1.0f;
    w[k] = 0;
    m[k] = on[k] ? sm.dbm[rA + k * HS][0] : 0u;
  }
  for (;;) {
    int ix[HPT][D];
    bool any = false;
#pragma unroll
    for (int k = 0; k < HPT; k++)
#pragma unroll
      for (int q = 0; q < D; q++) {
        while (on[k] && !m[k] && w[k] < 7) m[k] = sm.dbm[rA + k * HS][++w[k]];
        ix[k][q] = m[k] ? w[k] * 32 + __ffs(m[k]) - 1 : -1;
        m[k] &= m[k] - 1;
        any |= ix[k][q] >= 0;
      }
    if (!any) break;
    float v[HPT][D];
#pragma unroll
    for (int k = 0; k < HPT; k++)
#pragma unroll
      for (int q = 0; q < D; q++) v[k][q] = ix[k][q] >= 0 ? S[k][ix[k][q] * VD] : 0.0f;
#pragma unroll
    for (int k = 0; k < HPT; k++)
#pragma unroll
      for (int q = 0; q < D; q++) {
        const float nv = lx_mul(v[k][q], e[k]);
        if (ix[k][q] >= 0) S[k][ix[k][q] * VD] = nv;
        const unsigned nzb = __ballot_sync(0xffffffffu, ix[k][q] >= 0 && nv != 0.0f);
        if (lane == 0 && nzb)
          atomicOr(&sm.nzm[rA + k * HS][ix[k][q] >> 5], 1u << (ix[k][q] & 31));
      }
  }
}

__device__ __forceinline__ void item_decay(Smem& sm, float* S0) {
  const int t = threadIdx.x, lane = t & 31, grp = t >> 7;
  constexpr int D = 8;
  const uint32_t msel = 0x11111111u << grp;
  int h = 0, w = 0;
  uint32_t m = sm.ge[0] != 1.0f ? (sm.dbm[0][0] & msel) : 0u;
  for (;;) {
    int ix[D];  // head * KD + row, or -1
    bool any = false;
#pragma unroll
    for (int q = 0; q < D; q++) {
      while (!m && h < R) {
        if (++w == 8) {
          w = 0;
          if (++h == R) break;
          if (sm.ge[h] == 1.0f) {  // this head does not decay now: its bitmap stays
            w = 7;
            continue;
          }
        }
        m = sm.dbm[h][w] & msel;
      }
      ix[q] = m ? h * KD + w * 32 + __ffs(m) - 1 : -1;
      m &= m - 1;
      any |= ix[q] >= 0;
    }
    if (!any) break;
    float v[D];
#pragma unroll
    for (int q = 0; q < D; q++) v[q] = ix[q] >= 0 ? S0[(size_t)ix[q] * VD] : 0.0f;
#pragma unroll
    for (int q = 0; q < D; q++) {
      const int hh = ix[q] >= 0 ? ix[q] / KD : 0, row = ix[q] & (KD - 1);
      const float nv = lx_mul(v[q], sm.ge[hh]);
      if (ix[q] >= 0) S0[(size_t)ix[q] * VD] = nv;
      // the warp's 32 columns of the row (its rows are the same on every lane)
      const unsigned nzb = __ballot_sync(0xffffffffu, ix[q] >= 0 && nv != 0.0f);
      if (lane == 0 && nzb) atomicOr(&sm.nzm[hh][row >> 5], 1u << (row & 31));
    }
  }
}

// the key's delta-rule write into value head r (S at row 0, column j), after the decay
__device__ __forceinline__ void item_write(Smem& sm, float* S, int r, int j, int nk) {
  if (nk) {
    float kv = 0.0f;
    for (int a0 = 0; a0 < nk; a0 += 8) {
      float hv[8];
#pragma unroll
      for (int q = 0; q < 8; q++) hv[q] = a0 + q < nk ? S[sm.kidx[a0 + q] * VD] : 0.0f;
#pragma unroll
      for (int q = 0; q < 8; q++)
        if (a0 + q < nk) kv = lx_add(kv, lx_mul(hv[q], sm.kval[a0 + q]));
    }
    const float delta = lx_mul(lx_sub(sm.buf[2 * KD + r * VD + j], kv), sm.beta[r]);
    for (int a = 0; a < nk; a++) {
      float* hp = S + sm.kidx[a] * VD;
      *hp = lx_add(*hp, lx_mul(sm.kval[a], delta));
    }
  }
}

// Qwen3_5RMSNormGated of value head r (one warp, lane: columns lane + 32 q) whose o is not all
// zero: bf16(bf16(w * bf16(o * rsqrt(mean(o^2) + eps))) * silu(z)), z = bf16(in_proj_z . x)
__device__ __forceinline__ void item_out(const Dev& P, Smem& sm, const unsigned char* B,
                                      const lxb_bitem& bi, int r, const uint16_t* w_in,
                                      float r_in) {
  const int lane = threadIdx.x & 31;
  const float* o = sm.ob[r];
  const float o0 = o[4 * lane], o1 = o[4 * lane + 1], o2 = o[4 * lane + 2], o3 = o[4 * lane + 3];
  const int32_t* zp = reinterpret_cast<const int32_t*>(B + bi.z);
  const uint32_t* ze = reinterpret_cast<const uint32_t*>(B + bi.z + ((4 * 1025 + 15) & ~15));
  float sq = lx_mul(o0, o0);
  sq = lx_add(sq, lx_mul(o1, o1));
  sq = lx_add(sq, lx_mul(o2, o2));
  sq = lx_add(sq, lx_mul(o3, o3));
  sq = warp_xor_sum(sq);
  const float rr = lx_rsqrt(lx_add(lx_div(sq, 128.0f), P.eps));
  const uint16_t* gw = reinterpret_cast<const uint16_t*>(B + bi.prm) + 2 * R;
  uint16_t* on = sm.on[bi.slot];
#pragma unroll 1
  for (int q = 0; q < 4; q++) {
    const int j = lane + 32 * q;
    const int zr = r * VD + j;
    const float z = xrow_dot(sm, ze + zp[zr], zp[zr + 1] - zp[zr], w_in, r_in);
    const float hn = lx_rbf(lx_mul(o[j], rr));
    const float u = lx_rbf(lx_mul(lx_f(gw[j]), hn));
    on[r * VD + j] = lx_rb(lx_mul(u, d_silu(lx_rbf(z))));
  }
  if (lane == 0) atomicOr(&sm.vhmask[bi.slot], 1u << r);
}

// the query's and key's l2 norms (warp 0; lane 0 the query's, lane 1 the key's), in place
__device__ __forceinline__ void qk_norm(Smem& sm, int nq, int nk) {
  const int lane = threadIdx.x & 31;
  float inv = 0.0f;
  if (lane == 0 && nq) inv = l2_inv(sm.qval, nq);
  if (lane == 1 && nk) inv = l2_inv(sm.kval, nk);
  const float iq = __shfl_sync(0xffffffffu, inv, 0), ik = __shfl_sync(0xffffffffu, inv, 1);
  if (lane < nq) sm.qval[lane] = lx_mul(lx_rbf(lx_mul(sm.qval[lane], iq)), 0.0625f);
  if (lane < nk) sm.kval[lane] = lx_rbf(lx_mul(sm.kval[lane], ik));
}

// An item's end, after o is in sm.ob: the bitmaps of the rows a key wrote, then the gated norm
// per value head with output (warp r); a head without out_proj entries has no z rows staged and
// cannot write: it skips this. Returns whether the item wrote.
__device__ __forceinline__ bool item_tail(const Dev& P, Smem& sm, const unsigned char* B,
                                          const lxb_bitem& bi, uint32_t* bm, int nk,
                                          const uint16_t* w_in, float r_in) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  __syncthreads();
  if ((bi.flags & LXB_IT_DECAYS) && t < R) {  // rows the key wrote may now be nonzero
    uint32_t* b = bm + (bi.kh * R + t) * 8;
    for (int a = 0; a < nk; a++) b[sm.kidx[a] >> 5] |= 1u << (sm.kidx[a] & 31);
  }
  if (warp < R && bi.z >= 0) {
    const float* o = sm.ob[warp];
    const bool nz = __any_sync(0xffffffffu, o[4 * lane] != 0.0f || o[4 * lane + 1] != 0.0f ||
                                                o[4 * lane + 2] != 0.0f || o[4 * lane + 3] != 0.0f);
    if (nz) item_out(P, sm, B, bi, warp, w_in, r_in);
  }
  __syncthreads();
  return sm.vhmask[bi.slot] != 0 && (bi.flags & LXB_IT_OUT);
}

// B: the step blob (shared memory); bi: this item's record in it; w_in: the staged input norm.
// lmeta / lold (a group step's layer after its first, "speculative"): where to log the item's
// window shifts (meta: window index | item << 10 | lrel << 12), and a key firing or a decay is
// not done but reported. Returns ITEM_DONE, ITEM_WROTE (some value head has output and the head
// has out_proj entries), ITEM_PENDING (speculative and heavy: its windows shifted and logged,
// nothing else done) or ITEM_UNTOUCHED (speculative and not loggable: nothing done).
enum { ITEM_DONE = 0, ITEM_WROTE = 1, ITEM_PENDING = 2, ITEM_UNTOUCHED = 3 };
__device__ int gdn_item(const Dev& P, const Run& run, Smem& sm, const unsigned char* B,
                        const lxb_bitem& bi, float* rec, uint16_t* conv, uint32_t* bm, int s,
                        int L, int step, const uint16_t* w_in, float r_in, uint32_t* lmeta,
                        uint2* lold, uint32_t lmark) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const bool spec = lmeta != nullptr;
  if (spec && (bi.n_eager > 32 || (bi.flags & LXB_IT_NONRES))) return ITEM_UNTOUCHED;
  if (t == 0) sm.drows = 0;  // (read after the barriers below)
  const uint4* ch = reinterpret_cast<const uint4*>(B + bi.eager);
  // the eager rows' products, all entries at once over the block (the entries of the item's
  // eager channels are contiguous in the blob, in channel order); whether any is nonzero comes
  // with the barrier after them
  uint32_t e_first = 0;
  bool pre = false, zin = false;
  if (bi.n_eager > 0) {
    e_first = ch[0].x;
    const uint4 al = ch[2 * (bi.n_eager - 1)];
    const int ntot = (int)((al.x + 4u * (al.y & 0xffffu) - e_first) / 4u);
    if (ntot <= LXB_MAXPROD) {
      const uint32_t* E = reinterpret_cast<const uint32_t*>(B + e_first);
      bool nz = false;
      for (int k = t; k < ntot; k += NT) {
        const float p = lx_mul(xn_at(sm, w_in, r_in, E[k] & 0xffffu), lx_f((uint16_t)(E[k] >> 16)));
        sm.prod[k] = p;
        nz |= p != 0.0f;
      }
      zin = !__syncthreads_or(nz);
      pre = true;
    }
  }
  if (bi.n_eager <= 32) {
    // one warp: the channels in ascending order (queries, then keys), compacted by ballot
    if (warp == 0) {
      float v = 0.0f;
      int slot = 0;
      if (lane < bi.n_eager) {
        const uint4 a = ch[2 * lane], b = ch[2 * lane + 1];
        if (spec) {  // the window before the shift (resident: LXB_IT_NONRES is clear)
          lmeta[lane] = b.y | lmark;
          lold[lane] = sm.win[b.y];
        }
        v = eager_channel(sm, B, a, b, conv, w_in, r_in,
                          pre ? sm.prod + (a.x - e_first) / 4u : nullptr, zin);
        slot = (int)(a.y >> 16);
      }
      const bool nz = lane < bi.n_eager && v != 0.0f;
      const unsigned mq = __ballot_sync(0xffffffffu, nz && slot < KD);
      const unsigned mk = __ballot_sync(0xffffffffu, nz && slot >= KD);
      if (nz) {
        const unsigned m = slot < KD ? mq : mk;
        const int k = __popc(m & ((1u << lane) - 1u));
        if (slot < KD) {
          sm.qidx[k] = slot;
          sm.qval[k] = v;
        } else {
          sm.kidx[k] = slot - KD;
          sm.kval[k] = v;
        }
      }
      __syncwarp();
      const int nq = __popc(mq), nk = __popc(mk);
      if (lane == 0) {  // the lists' l2 norms come after the block barrier (qk_norm)
        sm.nq = nq;
        sm.nk = nk;
        sm.qkn = 0;
        sm.vhmask[bi.slot] = 0;
        sm.vhlay[bi.slot] = L;
        sm.vhtok[bi.slot] = step;
      }
    }
  } else {
    eager_block(sm, B, bi, conv, w_in, r_in, pre ? sm.prod : nullptr, e_first, zin);
    if (t == 0) {
      sm.vhlay[bi.slot] = L;
      sm.vhtok[bi.slot] = step;
    }
  }
  // warp 1: g, only for a head that can decay (for the others softplus underflows to zero
  // whatever the input: g is 0, as the table builder proved); beta only when a key fires
  if (warp == 1 && lane < R)
    sm.g[lane] = (bi.flags & LXB_IT_DECAYS) ? item_g(sm, B, bi, lane, w_in, r_in) : 0.0f;
  __syncthreads();
  // a head without out_proj entries: its readout has no use (nothing of it reaches the
  // residual), only a key's write and a decay change its state
  const int nq = (bi.flags & LXB_IT_OUT) ? sm.nq : 0, nk = sm.nk;
  int anyg = 0;
#pragma unroll
  for (int r = 0; r < R; r++) anyg |= sm.g[r] != 0.0f;
  if (!nq && !nk && !anyg) return ITEM_DONE;  // the state stays as it is and o = 0
  if (spec && (nk || anyg)) return ITEM_PENDING;  // a state write waits for its input to be final
  const bool normed = sm.qkn;
  if (nq && !nk && !anyg) {
    // a pure readout: its first rows' loads go out while warp 0 norms the query
    static_assert(NT / VD == 4 && R == 8, "two value heads per thread");
    const int j = t & (VD - 1);
    const int rA = t >> 7;
    const float* SA = rec + (size_t)(bi.kh * R + rA) * KD * VD + j;
    const float* SB = SA + (size_t)4 * KD * VD;
    float hA[8], hB[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const bool ok = q < nq;
      const int ix = ok ? sm.qidx[q] : 0;
      hA[q] = ok ? SA[ix * VD] : 0.0f;
      hB[q] = ok ? SB[ix * VD] : 0.0f;
    }
    if (!normed && warp == 0) qk_norm(sm, nq, 0);
    __syncthreads();
    float oA = 0.0f, oB = 0.0f;
#pragma unroll
    for (int q = 0; q < 8; q++)
      if (q < nq) {
        const float qv = sm.qval[q];
        oA = lx_add(oA, lx_mul(hA[q], qv));
        oB = lx_add(oB, lx_mul(hB[q], qv));
      }
    for (int a0 = 8; a0 < nq; a0 += 8) {
#pragma unroll
      for (int q = 0; q < 8; q++) {
        const bool ok = a0 + q < nq;
        const int ix = ok ? sm.qidx[a0 + q] : 0;
        hA[q] = ok ? SA[ix * VD] : 0.0f;
        hB[q] = ok ? SB[ix * VD] : 0.0f;
      }
#pragma unroll
      for (int q = 0; q < 8; q++)
        if (a0 + q < nq) {
          const float qv = sm.qval[a0 + q];
          oA = lx_add(oA, lx_mul(hA[q], qv));
          oB = lx_add(oB, lx_mul(hB[q], qv));
        }
    }
    sm.ob[rA][j] = lx_rbf(oA);
    sm.ob[rA + 4][j] = lx_rbf(oB);
    return item_tail(P, sm, B, bi, bm, 0, w_in, r_in) ? ITEM_WROTE : ITEM_DONE;
  }
  if (!normed) {
    if (warp == 0) qk_norm(sm, nq, nk);
    __syncthreads();
  }
  if (anyg && t < R * 8) {  // the decaying heads' nonzero-row bitmaps, for item_decay
    const uint32_t word = bm[(bi.kh * R + (t >> 3)) * 8 + (t & 7)];
    sm.dbm[t >> 3][t & 7] = word;
    sm.nzm[t >> 3][t & 7] = 0u;
    const float g = sm.g[t >> 3];
    const float e = g != 0.0f ? lx_exp(g) : 1.0f;
    if ((t & 7) == 0) sm.ge[t >> 3] = e;
    const int n = e != 1.0f ? __popc(word) : 0;  // (warps 0 and 1: the 64 words)
    const int wn = __reduce_add_sync(0xffffffffu, n);
    if (lane == 0) atomicAdd(&sm.drows, wn);
  }
  if (nk) item_fire(P, run, sm, B, bi, conv, s, L, step, w_in, r_in);  // (ends with a barrier)
  else if (anyg) __syncthreads();
  // the delta rule, thread = (state column j, value heads rA and rA + 4): the decay and the
  // key's write per head (rare), then both heads' readouts with their loads in flight together
  static_assert(NT / VD == 4 && R == 8, "two value heads per thread");
  {
    const int j = t & (VD - 1);
    const int rA = t >> 7;
    float* SA = rec + (size_t)(bi.kh * R + rA) * KD * VD + j;
    float* SB = SA + (size_t)4 * KD * VD;
    if (anyg) {
      if (sm.drows > 128) item_decay(sm, rec + (size_t)bi.kh * R * KD * VD + j);
      else item_decay_pairs(sm, SA, SB, rA);
      __syncthreads();  // the decay's rows are shared out over the block: all of it done first,
                        // then a decayed head's bitmap (the rows still nonzero; keys add theirs)
      if (t < R * 8 && sm.ge[t >> 3] != 1.0f)
        bm[(bi.kh * R + (t >> 3)) * 8 + (t & 7)] = sm.nzm[t >> 3][t & 7];
    }
    if (nk) {
      item_write(sm, SA, rA, j, nk);
      item_write(sm, SB, rA + 4, j, nk);
    }
    float oA = 0.0f, oB = 0.0f;
    for (int a0 = 0; a0 < nq; a0 += 8) {
      float hA[8], hB[8];
#pragma unroll
      for (int q = 0; q < 8; q++) {
        const bool ok = a0 + q < nq;
        const int ix = ok ? sm.qidx[a0 + q] : 0;
        hA[q] = ok ? SA[ix * VD] : 0.0f;
        hB[q] = ok ? SB[ix * VD] : 0.0f;
      }
#pragma unroll
      for (int q = 0; q < 8; q++)
        if (a0 + q < nq) {
          const float qv = sm.qval[a0 + q];
          oA = lx_add(oA, lx_mul(hA[q], qv));
          oB = lx_add(oB, lx_mul(hB[q], qv));
        }
    }
    sm.ob[rA][j] = lx_rbf(oA);
    sm.ob[rA + 4][j] = lx_rbf(oB);
  }
  return item_tail(P, sm, B, bi, bm, nk, w_in, r_in) ? ITEM_WROTE : ITEM_DONE;
}

// A query/key channel's projection by one thread: its in_proj_qkv row's products (the input
// norm taken per column, weights w) summed in entry order from +0, the same sum as
// eager_channel's; the entries e (column | bf16 << 16) staged or in global memory
__device__ __forceinline__ float chan_sum(const Smem& sm, const uint32_t* e, int ne,
                                          const uint16_t* w, float r) {
  float ps = 0.0f;
  for (int k = 0; k < ne; k += 8) {  // 8 entries' loads in flight, then the sum in order
    uint32_t en[8];
#pragma unroll
    for (int q = 0; q < 8; q++) en[q] = k + q < ne ? e[k + q] : 0u;
    float pv[8];
#pragma unroll
    for (int q = 0; q < 8; q++)
      pv[q] = k + q < ne ? lx_mul(xn_at(sm, w, r, en[q] & 0xffffu), lx_f((uint16_t)(en[q] >> 16)))
                         : 0.0f;
#pragma unroll
    for (int q = 0; q < 8; q++)
      if (k + q < ne) ps = lx_add(ps, pv[q]);
  }
  return ps;
}

// A query/key channel evaluated from the global tables (its entries in the entry pool, the input
// norm's weights w in the u16 pool), the window left as it is (nw: the shifted one)
__device__ __forceinline__ float quiet_chan(const Dev& P, const Smem& sm, const lxb_chan& c,
                                            const uint16_t* w, float r, const uint2 win, uint2& nw) {
  return conv_step(win, lx_rb(chan_sum(sm, P.ent + c.ent, c.n, w, r)), c.t01, c.t23, nw);
}

// A group step's quiet pass over layers [l0, qhi), qhi = min(hi, l0 + LXB_QLAYERS) (returned):
// every item of this CTA in those layers at once, a thread per query/key channel. An item that
// cannot decay and whose key outputs are all zero (and query outputs too, if its head has
// out_proj entries) changes nothing but its windows (gdn_item would return at its first check):
// they are shifted here, logged for the undo when the layer is after lo (the step's first), and
// the item is done. Every other item (one that is not resident, has more than 32 such channels,
// may decay, has a nonzero output, or finds no room in the log or the block) is left as it was,
// for the walk: sm.qfull, and vis (bit b: layer l0 + b has such items). Also the layers' ring
// rows of this step. Ends with a block barrier.
__device__ int quiet_pass(const Dev& P, const Run& run, Smem& sm, int s, int rank, int lo, int l0,
                          int hi, int step, float r, uint32_t& vis) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nl = max(0, min(hi, l0 + LXB_QLAYERS) - l0);
  if (warp == 0) {
    // lane: layer l0 + lane. Its items with channels, in (layer, item) order: the first ones that
    // fit the log and the block are this pass's (their log entries and threads contiguous)
    const int L = l0 + lane;
    int cnt = 0, need = 0, chn = 0;
    if (lane < nl)
      for (int k = 0; k < LXB_ITEMSLOTS && sm.qinfo[L][k] != LXB_QNONE; k++) {
        const uint32_t qi = sm.qinfo[L][k];
        const int n = (int)((qi >> 24) & 63u);
        if (qi == LXB_QFULL || !n) continue;  // (no channel: nothing to do)
        cnt++;
        need += L > lo ? n : 0;
        chn += n;
      }
    int cb = cnt, nb = need, hb = chn;  // inclusive scans over the lanes
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int c2 = __shfl_up_sync(0xffffffffu, cb, o), n2 = __shfl_up_sync(0xffffffffu, nb, o),
                h2 = __shfl_up_sync(0xffffffffu, hb, o);
      if (lane >= o) {
        cb += c2;
        nb += n2;
        hb += h2;
      }
    }
    int pos = cb - cnt, off = nb - need, coff = hb - chn, full = 0, acc = 0, end = 0, cend = 0;
    if (lane < nl)
      for (int k = 0; k < LXB_ITEMSLOTS && sm.qinfo[L][k] != LXB_QNONE; k++) {
        const uint32_t qi = sm.qinfo[L][k];
        if (qi == LXB_QFULL) {
          full |= 1 << k;
          continue;
        }
        const int n = (int)((qi >> 24) & 63u), nd = L > lo ? n : 0;
        if (!n) continue;
        if (off + nd <= LXB_LOGMAX && coff + n <= NT) {
          sm.qtask[pos] = make_uint4((uint32_t)k | (uint32_t)L << 8, (uint32_t)off, (uint32_t)coff, qi);
          acc++;
          end = off + nd;
          cend = coff + n;
        } else {
          full |= 1 << k;  // no room: the walk's
        }
        pos++;
        off += nd;
        coff += n;
      }
    if (lane < nl) sm.qfull[lane] = full;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc += __shfl_xor_sync(0xffffffffu, acc, o);
      end = max(end, __shfl_xor_sync(0xffffffffu, end, o));
      cend = max(cend, __shfl_xor_sync(0xffffffffu, cend, o));
    }
    if (lane == 0) {
      sm.qn = acc;  // (the accepted items are a prefix of the order)
      sm.qlog = end;
      sm.qnch = cend;
    }
  } else {
    // meanwhile the other warps: the layers' ring rows (each CTA its block; rank 0 the factor)
    const int per = P.blk / 2;
    for (int idx = t - 32; idx < nl * per; idx += NT - 32) {
      const int q = idx / per, k = idx - q * per;
      const size_t slot = ((size_t)s * P.n_layers + l0 + q) * 4 + (step & 3);
      const float* xv = sm.x + rank * P.blk + 2 * k;
      reinterpret_cast<uint32_t*>(run.ring + slot * H + rank * P.blk)[k] =
          (uint32_t)lx_rb(xv[0]) | ((uint32_t)lx_rb(xv[1]) << 16);
    }
    if (rank == 0 && t - 32 < nl)
      run.ring_r[((size_t)s * P.n_layers + l0 + (t - 32)) * 4 + (step & 3)] = r;
  }
  __syncthreads();
  // thread t: channel t of the pass (its item: the last whose first thread is <= t)
  const int nch = sm.qnch;
  uint4 q = make_uint4(0u, 0u, 0u, 0u);
  uint32_t wi = 0;
  uint2 old = make_uint2(0u, 0u), nw = make_uint2(0u, 0u);
  if (t < nch) {
    int a = 0, b = sm.qn - 1;
    while (a < b) {
      const int m = (a + b + 1) >> 1;
      if ((int)sm.qtask[m].z <= t) a = m;
      else b = m - 1;
    }
    q = sm.qtask[a];
    const int L = (int)((q.x >> 8) & 255u);
    const lxb_chan c = P.chans[(q.w & 0xffffffu) + (t - q.z)];
    wi = c.win;
    old = sm.win[wi];
    const float v = quiet_chan(P, sm, c, P.u16 + sm.layers[L].ln_in, r, old, nw);
    // (a query matters only to a head with out_proj entries)
    if (v != 0.0f && ((q.w & LXB_QOUT) || c.slot >= KD)) atomicOr(&sm.qfull[L - l0], 1 << (q.x & 255u));
  }
  __syncthreads();
  vis = __ballot_sync(0xffffffffu, lane < nl && sm.qfull[lane] != 0);
  if (t < nch) {
    const int k = (int)(q.x & 255u), L = (int)((q.x >> 8) & 255u), e = (int)q.y + (t - (int)q.z);
    if (!((sm.qfull[L - l0] >> k) & 1)) {  // quiet: the shift stands (undone if L > J)
      if (L > lo) {
        sm.lmeta[e] = wi | (uint32_t)k << 10 | (uint32_t)(L - lo) << 12;
        sm.lold[e] = old;
      }
      sm.win[wi] = nw;
    } else if (L > lo) {
      sm.lmeta[e] = LXB_NOLOG;
    }
  }
  __syncthreads();
  return l0 + nl;
}

// --- the owned rows ---------------------------------------------------------------------------
// The MLP over this CTA's rows: own[row] = bf16(x + bf16(sum_u h_u w_d)), h_u re-evaluated here;
// the units and entries are in the staged blob (m: its MLP part).
// With w_in (the staged input norm, r_in its factor), the blob's GDN items are checked on the way,
// a thread per query/key channel on the top threads while the units are summed: an item that
// cannot decay and whose key outputs (and query outputs, if its head has out_proj entries) are
// all zero is done here (its windows shifted). Returns the items that need gdn_item: the others
// (the same in every thread; sm.qbad cleared by the caller before a block barrier).
__device__ uint32_t mlp_owner(const Dev& P, Smem& sm, const unsigned char* B, const lxb_bmlp& m,
                              float* own, const uint16_t* w_in = nullptr, float r_in = 0.0f) {
  const int t = threadIdx.x;
  const lxb_bunit* units = reinterpret_cast<const lxb_bunit*>(B + m.units);
  uint32_t full = 0;  // items not taken here
  int qk = -1;        // this thread's item, and channel (qa, qb)
  uint4 qa = make_uint4(0u, 0u, 0u, 0u), qb = qa;
  bool qout = false;
  if (w_in) {
    const lxb_bhdr* bh = reinterpret_cast<const lxb_bhdr*>(B);
    int qn = 0;
    for (int k = 0; k < bh->n_items; k++) {
      const lxb_bitem* bi = reinterpret_cast<const lxb_bitem*>(B + bh->item[k]);
      if (bi->n_eager > 32 || (bi->flags & (LXB_IT_NONRES | LXB_IT_DECAYS))) full |= 1u << k;
      else qn += bi->n_eager;
    }
    int idx = t - (NT - qn);
    if (idx >= 0)
      for (int k = 0; k < bh->n_items; k++) {
        const lxb_bitem* bi = reinterpret_cast<const lxb_bitem*>(B + bh->item[k]);
        if ((full >> k) & 1) continue;
        if (idx < bi->n_eager) {
          const uint4* ch = reinterpret_cast<const uint4*>(B + bi->eager);
          qa = ch[2 * idx];
          qb = ch[2 * idx + 1];
          qout = (bi->flags & LXB_IT_OUT) != 0;
          qk = k;
          break;
        }
        idx -= bi->n_eager;
      }
  }
  // the gate and up entries of all units are contiguous in the blob: their products first, all
  // threads at once, into prod (the units' entries in order), then one thread per unit sums its
  // own products in order, so the sums are the sequential ones
  const int g0 = m.n_units ? units[0].g : 0;
  const int ne = m.n_units ? (units[m.n_units - 1].u + 4 * units[m.n_units - 1].nu - g0) / 4 : 0;
  const uint32_t* ent = reinterpret_cast<const uint32_t*>(B + g0);
  float* prod = sm.prod;
  if (ne <= LXB_MAXPROD) {
#pragma unroll 4
    for (int e = t; e < ne; e += NT)
      prod[e] = lx_mul(sm.xm[ent[e] & 0xffffu], lx_f((uint16_t)(ent[e] >> 16)));
    __syncthreads();
  }
  for (int u = t; u < m.n_units; u += NT) {
    const lxb_bunit un = units[u];
    float gs = 0.0f, us = 0.0f;
    if (ne <= LXB_MAXPROD) {
      // both sums in order, 8 products of each loaded at a time (the two chains interleave)
      const float* pg = prod + (un.g - g0) / 4;
      const float* pu = prod + (un.u - g0) / 4;
      const int nmax = max((int)un.ng, (int)un.nu);
      for (int k = 0; k < nmax; k += 8) {
        float vg[8], vu[8];
#pragma unroll
        for (int q = 0; q < 8; q++) {
          vg[q] = k + q < un.ng ? pg[k + q] : 0.0f;
          vu[q] = k + q < un.nu ? pu[k + q] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < 8; q++) {
          if (k + q < un.ng) gs = lx_add(gs, vg[q]);
          if (k + q < un.nu) us = lx_add(us, vu[q]);
        }
      }
    } else {
      const uint32_t* ge = reinterpret_cast<const uint32_t*>(B + un.g);
      const uint32_t* ue = reinterpret_cast<const uint32_t*>(B + un.u);
      for (int k = 0; k < un.ng; k++)
        gs = lx_add(gs, lx_mul(sm.xm[ge[k] & 0xffffu], lx_f((uint16_t)(ge[k] >> 16))));
      for (int k = 0; k < un.nu; k++)
        us = lx_add(us, lx_mul(sm.xm[ue[k] & 0xffffu], lx_f((uint16_t)(ue[k] >> 16))));
    }
    const float gg = lx_rbf(gs), uu = lx_rbf(us);
    const float act = lx_rbf(d_silu(gg));
    sm.hbuf[u] = lx_rbf(lx_mul(act, uu));
  }
  uint2 qnw = make_uint2(0u, 0u);
  if (qk >= 0) {  // an item's channel (a query matters only to a head with out_proj entries)
    const float v = conv_step(sm.win[qb.y],
                              lx_rb(chan_sum(sm, reinterpret_cast<const uint32_t*>(B + qa.x),
                                             (int)(qa.y & 0xffffu), w_in, r_in)),
                              qa.w, qb.x, qnw);
    if (v != 0.0f && (qout || (qa.y >> 16) >= KD)) atomicOr(&sm.qbad, 1u << qk);
  }
  if (t == 0) sm.nlong = 0;
  __syncthreads();
  const int r0 = m.r0;
  const int32_t* rp = reinterpret_cast<const int32_t*>(B + m.down_ptr);
  const uint32_t* de = reinterpret_cast<const uint32_t*>(B + m.down_ent);
  for (int k = t; k < m.nr; k += NT) {
    const float xv = sm.x[r0 + k];
    float res = xv;
    float sd = 0.0f;
    bool any = false;
    const int e1 = rp[k + 1];
    if (m.nlong && e1 - rp[k] > LXB_LONG) {  // a warp's, below (if the list has room)
      const int q = atomicAdd(&sm.nlong, 1);
      if (q < LXB_LONGROWS) {
        sm.lrows[q] = k;
        continue;
      }
    }
    for (int e = rp[k]; e < e1; e += 8) {  // 8 entries' loads in flight, then the sum in order
      uint32_t w[8];
      float hv[8];
#pragma unroll
      for (int q = 0; q < 8; q++) w[q] = e + q < e1 ? de[e + q] : 0u;
#pragma unroll
      for (int q = 0; q < 8; q++) hv[q] = e + q < e1 ? sm.hbuf[w[q] & 0xffffu] : 0.0f;
#pragma unroll
      for (int q = 0; q < 8; q++)
        if (hv[q] != 0.0f) {  // (0 past the row's end)
          sd = lx_add(sd, lx_mul(hv[q], lx_f((uint16_t)(w[q] >> 16))));
          any = true;
        }
    }
    if (any) res = lx_rbf(lx_add(xv, lx_rbf(sd)));
    own[k] = res;
  }
  if (m.nlong) __syncthreads();  // (otherwise nothing was deferred; the plan counted them)
  // the long rows, a warp each: 32 entries' products at once, summed in the entries' order
  const int nlong = m.nlong ? min(sm.nlong, LXB_LONGROWS) : 0;
  const int lane = t & 31;
  for (int j = t >> 5; j < nlong; j += NT / 32) {
    const int k = sm.lrows[j];
    const int a = rp[k], b = rp[k + 1];
    float sd = 0.0f;
    bool any = false;
    uint32_t w = a + lane < b ? de[a + lane] : 0u;
    for (int e0 = a; e0 < b; e0 += 32) {
      const uint32_t wn = e0 + 32 + lane < b ? de[e0 + 32 + lane] : 0u;  // the next
      const float hv = e0 + lane < b ? sm.hbuf[w & 0xffffu] : 0.0f;
      const float p = hv != 0.0f ? lx_mul(hv, lx_f((uint16_t)(w >> 16))) : 0.0f;
      unsigned msk = __ballot_sync(0xffffffffu, hv != 0.0f);
      any |= msk != 0u;
      while (msk) {
        const int l = __ffs(msk) - 1;
        msk &= msk - 1u;
        sd = lx_add(sd, __shfl_sync(0xffffffffu, p, l));
      }
      w = wn;
    }
    if (lane == 0) {
      const float xv = sm.x[r0 + k];
      own[k] = any ? lx_rbf(lx_add(xv, lx_rbf(sd))) : xv;
    }
  }
  const uint32_t bad = w_in ? sm.qbad : 0u;
  if (qk >= 0 && !((bad >> qk) & 1)) sm.win[qb.y] = qnw;  // a quiet item: its windows shift
  return full | bad;
}

// every owned MLP row [r0, r0 + nr) unchanged (no staged MLP tables)
__device__ void copy_owner(Smem& sm, int r0, int nr, float* own) {
  for (int k = threadIdx.x; k < nr; k += NT) own[k] = sm.x[r0 + k];
}

// out_proj over this CTA's rows, from the layer's items' outputs (gathered over DSMEM)
__device__ void out_owner(const Dev& P, Smem& sm, int L, const lxb_owner& ow,
                          int rank, int tok, float* own, cg::cluster_group& cluster) {
  const int t = threadIdx.x;
  if (t < LXB_NK) {
    const uint32_t ki = sm.kinfo[L][t];
    uint32_t m = 0;
    if (ki) {  // (a slot another layer's or token's item has set since holds none of this)
      const int slot = (int)(ki & 0xffu), cta = (int)((ki >> 8) & 0xffu);
      m = *cluster.map_shared_rank(&sm.vhmask[slot], cta);
      if (*cluster.map_shared_rank(&sm.vhlay[slot], cta) != L ||
          *cluster.map_shared_rank(&sm.vhtok[slot], cta) != tok)
        m = 0;
    }
    sm.kmask[t] = (int)m;
  }
  if (t == 0) sm.nlong = 0;  // (the long rows' list, below)
  __syncthreads();
  // copy the active items' outputs: 16 key heads x 128 uint4
  for (int k = t; k < LXB_NK * (R * VD / 8); k += NT) {
    const int kh = k / (R * VD / 8), q = k % (R * VD / 8);
    if (!sm.kmask[kh]) continue;
    const uint32_t ki = sm.kinfo[L][kh];
    const uint4* src = reinterpret_cast<const uint4*>(
        cluster.map_shared_rank(&sm.on[ki & 0xffu][0], (int)((ki >> 8) & 0xffu)));
    reinterpret_cast<uint4*>(&sm.onall[kh][0])[q] = src[q];
  }
  __syncthreads();
  const int r0 = rank * P.blk;
  const int32_t* rp = ow.orow >= 0 ? P.i32 + ow.orow : nullptr;
  for (int k = t; k < P.blk; k += NT) {
    const float xv = sm.x[r0 + k];
    float res = xv;
    if (rp) {
      const int a = rp[k], b = rp[k + 1];
      if (ow.nlong && b - a > LXB_LONG) {  // a warp's, below (if the list has room)
        const int q = atomicAdd(&sm.nlong, 1);
        if (q < LXB_LONGROWS) {
          sm.lrows[q] = k;
          continue;
        }
      }
      float s = 0.0f;
      bool any = false;
      for (int e = a; e < b; e += 8) {
        uint32_t w[8];
#pragma unroll
        for (int q = 0; q < 8; q++) w[q] = e + q < b ? __ldg(P.ent + e + q) : 0u;
#pragma unroll
        for (int q = 0; q < 8; q++) {
          if (e + q >= b) continue;
          const uint32_t vd = w[q] & 0xffffu;
          const int kh = (int)(vd >> 10);
          if (!((sm.kmask[kh] >> ((vd >> 7) & 7)) & 1)) continue;
          const float ov = lx_f(sm.onall[kh][vd & 1023u]);
          if (ov != 0.0f) {
            s = lx_add(s, lx_mul(ov, lx_f((uint16_t)(w[q] >> 16))));
            any = true;
          }
        }
      }
      if (any) res = lx_rbf(lx_add(xv, lx_rbf(s)));
    }
    own[k] = res;
  }
  if (!ow.nlong) return;  // (the plan counted them: nothing was deferred)
  __syncthreads();
  // the long rows, a warp each: 32 entries' loads and products at once, then their sum in the
  // entries' order (the same additions as one thread's, in the same order: the same bits)
  const int nlong = min(sm.nlong, LXB_LONGROWS);
  const int lane = t & 31;
  for (int j = t >> 5; j < nlong; j += NT / 32) {
    const int k = sm.lrows[j];
    const int a = rp[k], b = rp[k + 1];
    float s = 0.0f;
    bool any = false;
    uint32_t w = a + lane < b ? __ldg(P.ent + a + lane) : 0u;
    for (int e0 = a; e0 < b; e0 += 32) {
      const uint32_t wn = e0 + 32 + lane < b ? __ldg(P.ent + e0 + 32 + lane) : 0u;  // the next
      float p = 0.0f;
      bool nz = false;
      if (e0 + lane < b) {
        const uint32_t vd = w & 0xffffu;
        const int kh = (int)(vd >> 10);
        if ((sm.kmask[kh] >> ((vd >> 7) & 7)) & 1) {
          const float ov = lx_f(sm.onall[kh][vd & 1023u]);
          if (ov != 0.0f) {
            p = lx_mul(ov, lx_f((uint16_t)(w >> 16)));
            nz = true;
          }
        }
      }
      unsigned m = __ballot_sync(0xffffffffu, nz);
      any |= m != 0u;
      while (m) {
        const int l = __ffs(m) - 1;
        m &= m - 1u;
        s = lx_add(s, __shfl_sync(0xffffffffu, p, l));
      }
      w = wn;
    }
    if (lane == 0) {
      const float xv = sm.x[r0 + k];
      own[k] = any ? lx_rbf(lx_add(xv, lx_rbf(s))) : xv;
    }
  }
}

// The owner's rows into every CTA's push buffer of this parity, as bf16 (the residual's values
// are bf16; 16-byte DSMEM stores before the step's cluster barrier, which makes them visible);
// own must be complete (a block barrier after it was written).
__device__ void push_rows(const Dev& P, Smem& sm, const float* own, int par, int r0, int nr,
                          cg::cluster_group& cluster) {
  const int per = nr / 8;  // uint4 (8 rows) per destination
  for (int k = threadIdx.x; k < per * P.C; k += NT) {
    const int d = k / per, q = k % per;
    const float* o = own + 8 * q;
    const uint4 v = make_uint4((uint32_t)lx_rb(o[0]) | ((uint32_t)lx_rb(o[1]) << 16),
                               (uint32_t)lx_rb(o[2]) | ((uint32_t)lx_rb(o[3]) << 16),
                               (uint32_t)lx_rb(o[4]) | ((uint32_t)lx_rb(o[5]) << 16),
                               (uint32_t)lx_rb(o[6]) | ((uint32_t)lx_rb(o[7]) << 16));
    uint4* dst = reinterpret_cast<uint4*>(cluster.map_shared_rank(&sm.xin[par][r0], d));
    dst[q] = v;
  }
}

// The replica's rows [lo, hi) from the push buffer (after the cluster barrier; the others did not
// change), with the residual's sum of squares in the canonical order on the way (lane t: the
// squares of x[t + 512 i], i = 0..4, in order, then the two butterflies): the norm factor
__device__ float take_rows_norm(const Dev& P, Smem& sm, int par, int lo = 0, int hi = H) {
  static_assert(H == 5 * NT, "five residual rows per thread");
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 5; i++) {
    const int c = t + NT * i;
    float v;
    if (c >= lo && c < hi) {
      v = lx_f(sm.xin[par][c]);
      sm.x[c] = v;
    } else {
      v = sm.x[c];
    }
    s = i == 0 ? lx_mul(v, v) : lx_add(s, lx_mul(v, v));
  }
  s = warp_xor_sum(s);
  if (lane == 0) sm.red[warp] = s;
  __syncthreads();
  float v = lane < 16 ? sm.red[lane] : 0.0f;
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) v = lx_add(v, __shfl_xor_sync(0xffffffffu, v, off));
  return norm_factor(P, __shfl_sync(0xffffffffu, v, 0));
}

__device__ void load_embed(const Run& run, const Dev& P, Smem& sm, int tok) {
  const uint4* e = reinterpret_cast<const uint4*>(run.embed + ((int64_t)tok + P.offset) * H);
  for (int k = threadIdx.x; k < H / 8; k += NT) {
    const uint4 v = __ldg(e + k);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      sm.x[8 * k + 2 * q] = lx_f((uint16_t)(w[q] & 0xffffu));
      sm.x[8 * k + 2 * q + 1] = lx_f((uint16_t)(w[q] >> 16));
    }
  }
  __syncthreads();
}

// The head's per-group tables from sm.xm: htg[g][code] = the sum, in column order from +0, of the
// group's 4 dense columns' weights (by their 2-bit codes) times xm. Ends with a block barrier.
// Returns (in every thread) whether xm is nonzero in some column with sparse entries: if not,
// every sparse product is +-0 and a row's sparse sum stays +0, so head_rows skips the entries
// (as the reference visits only sparse columns with x != 0, lx/csrc/mega.cu:584-595).
__device__ int head_tables(const Dev& P, Smem& sm) {
  const int nd = P.n_dense, ng = (nd + 3) / 4;
  for (int k = threadIdx.x; k < ng * 256; k += NT) {
    const int g = k >> 8, code = k & 255;
    float s = 0.0f;
    for (int j = 0; j < 4 && 4 * g + j < nd; j++)
      s = lx_add(s, lx_mul(P.htab[(code >> (2 * j)) & 3], sm.xm[P.dense_cols[4 * g + j]]));
    sm.htg[g][code] = s;
  }
  int any = 0;
#pragma unroll
  for (int i = 0; i < H / NT; i++) {
    const int c = threadIdx.x + NT * i;
    any |= ((sm.hspm[c >> 5] >> (c & 31)) & 1u) && sm.xm[c] != 0.0f;
  }
  return __syncthreads_or(any);
}

// The head rows of one part, into this thread's running first maximum (bv, bi) of the bf16 logits
// (a thread's rows ascend within a part, and parts are visited in ascending order).
__device__ void head_rows(const Dev& P, const Smem& sm, const lxb_headcta hc, int hsp, float& bv,
                          int& bi) {
  const int t = threadIdx.x;
  const int nd = P.n_dense, ng = (nd + 3) / 4;
  const int32_t* rp = P.i32 + hc.rowptr;
  // any sparse entry in these rows, and a nonzero input in some sparse column (head_tables)
  const bool sparse = hsp && rp[0] != rp[hc.r1 - hc.r0];
  constexpr int U = 4;  // rows in flight per thread
  for (int row0 = hc.r0 + t; row0 < hc.r1; row0 += NT * U) {
    uint64_t code[U];
#pragma unroll
    for (int q = 0; q < U; q++) {
      const int row = row0 + q * NT;
      code[q] = (row < hc.r1 && nd) ? __ldg(P.hcodes + row) : 0ull;
    }
    // the dense part, groups in order per row; the table loads of all rows and groups are
    // independent of the sums, so they are all in flight together
    float tv[U][LXB_MAXDENSE / 4];
#pragma unroll
    for (int g = 0; g < LXB_MAXDENSE / 4; g++)
#pragma unroll
      for (int q = 0; q < U; q++)
        tv[q][g] = g < ng ? sm.htg[g][(code[q] >> (8 * g)) & 255u] : 0.0f;
#pragma unroll
    for (int q = 0; q < U; q++) {
      const int row = row0 + q * NT;
      if (row >= hc.r1) continue;
      float D = 0.0f;
#pragma unroll
      for (int g = 0; g < LXB_MAXDENSE / 4; g++)
        if (g < ng) D = lx_add(D, tv[q][g]);
      float S = 0.0f;
      if (sparse) {
        const int ea = __ldg(rp + row - hc.r0), eb = __ldg(rp + row - hc.r0 + 1);
        for (int e = ea; e < eb; e++) {
          const uint32_t w = __ldg(P.ent + e);
          S = lx_add(S, lx_mul(lx_f((uint16_t)(w >> 16)), sm.xm[w & 0xffffu]));
        }
      }
      const float lg = lx_rbf(lx_add(D, S));
      if (lg > bv) {
        bv = lg;
        bi = row;
      }
    }
  }
}

// the first maximum over the block (larger value, then smaller row) into *ov_out / *oi_out
// (shared; by default sm.bestv / sm.besti, which other CTAs read after a cluster barrier)
__device__ void head_reduce(Smem& sm, float bv, int bi, float* ov_out = nullptr,
                            int* oi_out = nullptr) {
  const int t = threadIdx.x;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, bv, off);
    const int oi = __shfl_down_sync(0xffffffffu, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  const int lane = t & 31, warp = t >> 5;
  __syncthreads();
  if (lane == 0) {
    sm.red[warp] = bv;
    reinterpret_cast<int*>(sm.hbuf)[warp] = bi;
  }
  __syncthreads();
  if (t == 0) {
    for (int w = 1; w < NT / 32; w++) {
      const float ov = sm.red[w];
      const int oi = reinterpret_cast<int*>(sm.hbuf)[w];
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    *(ov_out ? ov_out : &sm.bestv) = bv;
    *(oi_out ? oi_out : &sm.besti) = bi;
  }
  __syncthreads();
}

// the first maximum of the cluster's CTAs' sm.bestv / sm.besti into sm.cv / sm.ci (every CTA the
// same), after a cluster barrier that follows their head_reduce; ends with a block barrier
__device__ void cluster_max(Smem& sm, cg::cluster_group& cluster, int C) {
  const int t = threadIdx.x;
  if (t < 32) {
    float bv = -LXB_INF;
    int bi = 0x7fffffff;
    if (t < C) {
      bv = *cluster.map_shared_rank(&sm.bestv, t);
      bi = *cluster.map_shared_rank(&sm.besti, t);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, bv, off);
      const int oi = __shfl_down_sync(0xffffffffu, bi, off);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (t == 0) {
      sm.cv = bv;
      sm.ci = bi;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// A head helper CTA (helper cluster hk = 1..n_help, rank c): the slices LXB_HEADMAIN + j of
// rank c's rows with j % n_help == hk - 1. Per token: wait for the decoding cluster's head input,
// take the first maximum over its slices, publish it. Every wait is bounded; a helper that gives
// up sets LXB_S_HELPER and leaves (the decoding cluster then takes its slices itself, so the
// stream stays exact).
__device__ void head_helper(const Dev& P, const Run& run, Smem& sm, int rank, int hk) {
  const int t = threadIdx.x;
  const int part = hk * P.C + rank;
  if (run.help_drill) return;
  const unsigned long long done = run.epoch | 0xffffffffull;
  for (int i = 0; i < run.n_tokens; i++) {
    const unsigned long long want = run.epoch | (unsigned long long)(i + 1);
    if (t == 0) {
      int go = 0;
      const long long t0 = clock64();
      for (;;) {
        const unsigned long long v = ld_acquire_u64(run.hseq);
        if (v == want) {
          go = 1;
          break;
        }
        if (v == done) break;
        if (clock64() - t0 > (1ll << 32)) {  // ~2 s: the decoding cluster is gone
          atomicOr(P.status, LXB_S_HELPER);
          break;
        }
        __nanosleep(64);
      }
      sm.tok = go;
    }
    __syncthreads();
    if (!sm.tok) return;
    for (int k = t; k < H / 4; k += NT)
      reinterpret_cast<float4*>(sm.xm)[k] = __ldcg(reinterpret_cast<const float4*>(run.hx) + k);
    __syncthreads();
    const int hsp = head_tables(P, sm);
    float bv = -LXB_INF;
    int bi = 0x7fffffff;
    for (int k = LXB_HEADMAIN + hk - 1; k < LXB_HEADSLICES; k += run.n_help)
      head_rows(P, sm, P.headcta[rank * LXB_HEADSLICES + k], hsp, bv, bi);
    head_reduce(sm, bv, bi);
    if (t == 0) {
      uint4* hp = run.hpart + part;
      hp->x = __float_as_uint(sm.bestv);
      hp->y = (uint32_t)sm.besti;
      hp->w = (uint32_t)(want >> 32);
      __threadfence();
      asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(&hp->z), "r"((uint32_t)want)
                   : "memory");
    }
  }
}

// At the launch's end: every lazily kept conv window of this CTA's items becomes what the stock
// steps would have left, [P(n-4), P(n-3), P(n-2), P(n-1)].
__device__ void materialize(const Dev& P, const Run& run, Smem& sm, int s, int rank, int n) {
  for (int L = 0; L < P.n_layers; L++) {
    const lxb_layer ly = P.layers[L];
    if (!ly.has_gdn) continue;
    uint16_t* conv =
        reinterpret_cast<uint16_t*>(run.state_ptrs[((size_t)s * P.n_layers + L) * 2 + 1]);
    for (int k = 0; k < ly.n_items; k++) {
      const lxb_item it = P.items[ly.item0 + k];
      if (it.cta != rank) continue;
      for (int c0 = it.n_eager; c0 < it.n_ch; c0 += LXB_NSLOT) {
        const int c1 = min(it.n_ch, c0 + LXB_NSLOT);
        lazy_proj(P, run, sm, it, conv, s, L, n - 4, INT_MIN, false, c0, c1, P.u16 + ly.ln_in);
        for (int c = c0 + threadIdx.x; c < c1; c += NT) {
          const uint32_t cc = __ldg(reinterpret_cast<const uint32_t*>(P.chans + it.ch0 + c) + 2);
          const int i = c - c0;
          *reinterpret_cast<uint2*>(conv + (size_t)cc * 4) =
              make_uint2((uint32_t)sm.lz.pw[0][i] | ((uint32_t)sm.lz.pw[1][i] << 16),
                         (uint32_t)sm.lz.pw[2][i] | ((uint32_t)sm.lz.pw[3][i] << 16));
        }
        __syncthreads();
      }
    }
  }
}

// --- the device typing queue ---------------------------------------------------------------
// The reference types a command into the model-alone machine from the host, a batch of at most
// RX_SLOTS bytes at a time (KEY0 for the batch's first byte, KEY for the others), only at a record
// boundary and only when the machine has read every byte typed so far; it sees both conditions
// only at launch ends (lx/lx/linux.py:254-289). Here every CTA of the decoding cluster applies
// the same rule after every token (each CTA computes the same, so no exchange is needed).
__device__ __forceinline__ int type_class(const Run& run, int tok) {
  return (tok >= 0 && tok < run.typing.n_class) ? run.typing.tclass[tok] : 0;
}
// an input token counted into the RX FIFO: a typed key enters it, an RX read leaves it
__device__ __forceinline__ void type_count(const Run& run, Smem& sm, int tok) {
  const int c = type_class(run, tok);
  if (c & LXB_T_TYPED) sm.tq_wait++;
  if (c & LXB_T_RX) sm.tq_wait--;
}
// the next input after the current one (sm.tok) whose prediction is bi
__device__ __forceinline__ int type_next(const Run& run, Smem& sm, int s, int bi) {
  const lxb_typing& ty = run.typing;
  const int nk = ty.n_keys[s];
  if (sm.tq_left == 0 && sm.tq_k < nk && sm.tq_wait == 0 &&
      (type_class(run, sm.tok) & LXB_T_FINAL)) {
    sm.tq_left = min(ty.rx_slots, nk - sm.tq_k) - 1;  // this batch's keys after the first
    return ty.key0_base + ty.keys[(size_t)s * ty.max_keys + sm.tq_k++];
  }
  if (sm.tq_left > 0 && sm.tq_k < nk) {
    sm.tq_left--;
    return ty.key_base + ty.keys[(size_t)s * ty.max_keys + sm.tq_k++];
  }
  return bi;
}

__global__ void __launch_bounds__(NT, 1) lxb_decode_kernel(Dev P, Run run) {
  extern __shared__ __align__(128) unsigned char dsm[];
  Smem& sm = *reinterpret_cast<Smem*>(dsm);
  unsigned char* stage = dsm + ((sizeof(Smem) + 127) / 128) * 128;
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int C = P.C;
  const int s = blockIdx.x / C;
  const int t = threadIdx.x;
  // the head's sparse-column mask (read after the block barriers that precede every head step)
  for (int k = t; k < H / 32; k += NT) sm.hspm[k] = P.hsp ? P.hsp[k] : 0u;
  if (s >= run.n_streams) {  // a head helper cluster
    head_helper(P, run, sm, rank, s - run.n_streams + 1);
    return;
  }
  const int nsteps_tok = P.n_layers + 1;  // the layers, then the head
  if (t < 2) {
    sm.wflag[t] = 0;
    sm.gkey[t] = 0x7fffffff;
  }
  if (t == 0) sm.help_dead = 0;
  if (t == 0) {
    int tok = run.forced[(size_t)s * run.n_forced];
    if (tok < 0 || (int64_t)tok + P.offset >= P.n_embed_rows) {
      set_status(P, LXB_S_TOKEN, s, 0);
      tok = 0;
    }
    sm.tok = tok;
    if (run.typing.keys) {
      const int32_t* ts = run.typing.tstate + (size_t)s * 4;
      sm.tq_k = ts[0];
      sm.tq_wait = ts[1];
      sm.tq_left = ts[2];
      type_count(run, sm, tok);
    }
    sm.broken = 0;
    for (int b = 0; b < P.nbuf; b++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&sm.mbar[b])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // per-launch tables into shared memory: layer descriptors, this stream's state pointers, this
  // CTA's blob index, head rows and resident windows (pointers first: the windows use them)
  for (int k = t; k < P.n_layers * (int)(sizeof(lxb_layer) / 4); k += NT)
    reinterpret_cast<int*>(sm.layers)[k] = reinterpret_cast<const int*>(P.layers)[k];
  for (int k = t; k < 2 * P.n_layers; k += NT)
    (&sm.sptr[0][0])[k] = run.state_ptrs[(size_t)s * P.n_layers * 2 + k];
  for (int k = t; k <= P.n_layers; k += NT) sm.bref[k] = P.blobidx[k * C + rank];
  if (t == 0) {
    sm.win0 = P.winidx[2 * rank];
    sm.nwin = P.winidx[2 * rank + 1];
  }
  __syncthreads();
  for (int k = t; k < sm.nwin; k += NT) {  // the resident conv windows, from the state
    const int L = P.winmap[2 * (sm.win0 + k)], ch = P.winmap[2 * (sm.win0 + k) + 1];
    sm.win[k] = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(sm.sptr[L][1]) +
                                                (size_t)ch * 4);
  }
  for (int k = t; k < P.n_layers * LXB_ITEMSLOTS; k += NT) {  // this CTA's items per layer
    const int L = k / LXB_ITEMSLOTS, q = k % LXB_ITEMSLOTS;
    const unsigned char* Bg = P.blobs + sm.bref[L].off;
    const lxb_bhdr* bh = reinterpret_cast<const lxb_bhdr*>(Bg);
    uint32_t v = LXB_QNONE;
    if (q < bh->n_items) {
      const lxb_item it = P.items[reinterpret_cast<const lxb_bitem*>(Bg + bh->item[q])->item];
      v = (it.n_eager <= 32 && it.ch0 < (1 << 24) &&
           !(it.flags & (LXB_IT_NONRES | LXB_IT_DECAYS)))
              ? (uint32_t)it.ch0 | (uint32_t)it.n_eager << 24 | ((it.flags & LXB_IT_OUT) ? LXB_QOUT : 0u)
              : LXB_QFULL;
    }
    sm.qinfo[L][q] = v;
  }
  for (int k = t; k < P.n_layers * LXB_NK; k += NT) {  // every layer's items: slot and CTA
    const int L = k / LXB_NK, kh = k % LXB_NK;
    const int ii = P.i32[sm.layers[L].itemof + kh];
    uint32_t v = 0u;
    if (ii >= 0) {
      const lxb_item it = P.items[ii];
      v = (uint32_t)it.slot | (uint32_t)it.cta << 8 | 0x10000u;
    }
    sm.kinfo[L][kh] = v;
  }
  if (t == 0) sm.upm = 0ull;
  if (t < 64) {  // a lane per layer (from the plan's items: the same in every CTA)
    bool big = false;
    if (t < P.n_layers) {
      const lxb_layer& ly = sm.layers[t];
      big = ly.has_gdn && ly.n_items > 0;
      for (int k = 0; big && k < ly.n_items; k++) {
        const lxb_item it = P.items[ly.item0 + k];
        big = it.n_eager > 32 || (it.flags & (LXB_IT_NONRES | LXB_IT_DECAYS));
      }
    }
    const unsigned m = __ballot_sync(0xffffffffu, big);
    if ((t & 31) == 0) reinterpret_cast<unsigned*>(&sm.bigm)[t >> 5] = m;
  }
  if (t < LXB_ITEMSLOTS) {  // no slot holds an output yet
    sm.vhmask[t] = 0;
    sm.vhlay[t] = -1;
    sm.vhtok[t] = -1;
  }
  if (t == 0) stage_issue(P, sm, stage, 0, 0);  // step 0: layer 0
  __syncthreads();
  cluster.sync();  // every CTA's flags are initialised before anyone may push one
  int ph = 0;
  long long stp = 0;  // staged steps consumed
  uint32_t phases = 0u;  // bit b: the parity staging buffer b waits for next
  // the profile (thread 0's sections and counts, in shared memory: no registers held for them)
  if (t == 0)
    for (int k = 0; k < PR_N; k++) sm.pcs[k] = 0ull;
  long long c0 = clock64();
  const bool prof = run.prof != nullptr;
#define PROF(sec)                                     \
  do {                                                \
    if (prof && t == 0) {                             \
      const long long c1 = clock64();                 \
      sm.pcs[sec] += (unsigned long long)(c1 - c0);   \
      c0 = c1;                                        \
    }                                                 \
  } while (0)
#define COUNT(sec)                \
  do {                            \
    if (t == 0) sm.pcs[sec]++;    \
  } while (0)
  // the layer (or head, = n_layers) of global step k: k runs over the layers then the head
  int cur_layer = 0;  // the current step's layer (n_layers: the head)
  int cur_tok = 0;    // the current token
  int inflight = 0;   // the layer whose blob was issued last (-1: none), staged for the next take
  bool x_new = true;  // the residual changed since r_x was computed
  float r_x = 0.0f;   // the norm factor of the residual
  // the next step's blob into the free staging buffer (thread 0; the caller has synchronised
  // the block since the buffer's last use)
  // (issued by the last warp's first lane: that warp has the least work at the start of a step)
  auto issue_next = [&](long long cur) {
    if (cur_layer == P.n_layers && cur_tok == run.n_tokens - 1) {  // the launch's last step
      inflight = -1;
      return;
    }
    inflight = cur_layer + 1 == nsteps_tok ? 0 : cur_layer + 1;
    if (t == NT - 32 && !sm.broken)
      stage_issue(P, sm, stage, P.nbuf == 2 ? (int)((cur + 1) & 1) : 0, inflight);
  };
  // two buffers: make the copy staged for the next take layer Lnext's (a group step that starts
  // again at another layer): the copy in flight lands first, then Lnext's is issued in its place
  auto restage = [&](int Lnext) {
    if (inflight == Lnext) return;
    const int b = (int)(stp & 1);
    if (inflight >= 0) {
      unsigned long long polls = 0;
      const bool ok = !sm.broken && stage_wait(P, sm, b, (phases >> b) & 1u, s, cur_tok, polls);
      phases ^= 1u << b;
      if (!ok && t == 0) sm.broken = 1;
    }
    __syncthreads();  // every thread has seen that phase complete before the next one begins
    if (t == NT - 32 && !sm.broken) stage_issue(P, sm, stage, b, Lnext);
    inflight = Lnext;
  };
  // this step's blob: wait for it, and with two buffers start the next one's copy right away
  auto take = [&](int i) -> const unsigned char* {
    const int b = P.nbuf == 2 ? (int)(stp & 1) : 0;
    bool ok = !sm.broken;
    unsigned long long polls = 0;
    if (ok) ok = stage_wait(P, sm, b, (phases >> b) & 1u, s, i, polls);
    phases ^= 1u << b;
    if (prof && t == 0) sm.pcs[PR_POLLS] += polls;
    if (!ok && t == 0) sm.broken = 1;
    PROF(PR_WAIT);
    __syncthreads();
    PROF(PR_TAKESYNC);
    if (sm.broken) return nullptr;
    return sm.bsrc[b];
  };
  // A run of GDN-only layers [lo0, hi) as group steps, all on the residual as it was at the
  // step's start. That is exact as long as no layer before changes it. Each step first takes a
  // quiet pass over its layers (every item of this CTA at once: the ones whose query/key outputs
  // are all zero are done there), then walks the layers that still have items here, with no
  // cluster barrier between them: an item that writes (output) or one after the step's first
  // layer that would change its state (a key firing, a decay) ends the CTA's walk after that
  // layer and posts key 2 layer + (0 pending | 1 wrote) to every CTA's shared minimum; the
  // others stop before any later layer. After the barrier, with J the minimum's layer: the
  // window shifts of the layers after J (and of J's pending items) are undone from the log;
  // then either J again with only its pending items (as the first layer of the next group step)
  // or J's out_proj rows (the fix-up) and on from J + 1.
  int gp = 0;  // group steps so far (the key's parity)
  auto group_run = [&](const int lo0, const int hi, const int i) {
    int lo = lo0, rs_mask = 0, held_out = 0;
    bool resume = false;
    if (x_new) {
      r_x = norm_factor(P, block_ssq(sm, sm.x));
      x_new = false;
    }
    while (lo < hi) {
      const int gpar = gp & 1;
      if (t == 0) sm.gkey[gpar ^ 1] = 0x7fffffff;  // the next step's (nobody posts it before
                                                   // this step's barrier)
      const int l0 = resume ? lo + 1 : lo;  // (J's other items are done)
      uint32_t vis;  // the layers l0 + b that still have items here (the same in every thread)
      const int qhi = quiet_pass(P, run, sm, s, rank, lo, l0, hi, i, r_x, vis);
      PROF(PR_GITEMS);
      bool at_lo = resume && (rs_mask || held_out);  // J first: its pending items, its outputs
      auto peek = [&]() -> int { return at_lo ? lo : (vis ? l0 + __ffs(vis) - 1 : -1); };
      {
        const int f = peek();
        if (f >= 0) restage(f);
      }
      int nlog = sm.qlog, sL = -1, pend = 0, outL = 0;
      for (;;) {
        const int L = peek();
        if (L < 0) break;
        if (at_lo) at_lo = false;
        else vis &= vis - 1;
        const int want = (resume && L == lo) ? rs_mask : sm.qfull[L - l0];
        const bool held = resume && L == lo && held_out;  // J's outputs from the last step
        if (L > lo &&
            __syncthreads_or(t == 0 && *reinterpret_cast<volatile int*>(&sm.gkey[gpar]) < 2 * L))
          break;
        int st_any = held ? 1 : 0;
        if (want) {
          const lxb_layer& ly = sm.layers[L];
          cur_layer = L;
          restage(L);  // (in flight already, normally)
          const unsigned char* B = take(i);
          {  // the next layer with items here: its blob into the other buffer
            const int nx = peek();
            inflight = nx;
            if (nx >= 0 && t == NT - 32 && !sm.broken)
              stage_issue(P, sm, stage, (int)((stp + 1) & 1), nx);
          }
          PROF(PR_WAIT);
          const lxb_bhdr bh = B ? *reinterpret_cast<const lxb_bhdr*>(B) : lxb_bhdr{};
          float* rec = reinterpret_cast<float*>(sm.sptr[L][0]);
          uint16_t* conv = reinterpret_cast<uint16_t*>(sm.sptr[L][1]);
          uint32_t* bm = run.bitmaps + ((size_t)s * P.n_layers + L) * LXB_NV * 8;
          const float r = r_x;
          const uint16_t* w_in = (B && bh.ln_in >= 0)
                                     ? reinterpret_cast<const uint16_t*>(B + bh.ln_in)
                                     : P.u16 + ly.ln_in;
          if (B) {
            const lxb_bhdr* bhp = reinterpret_cast<const lxb_bhdr*>(B);  // (dynamic index: smem)
            for (int k = 0; k < bh.n_items; k++) {
              if (!((want >> k) & 1)) continue;  // done already
              const lxb_bitem bi = *reinterpret_cast<const lxb_bitem*>(B + bhp->item[k]);
              const bool spec = L > lo;
              if (spec && nlog + bi.n_eager > LXB_LOGMAX) {  // no room to undo: wait for J = L
                pend |= want & ~((1 << k) - 1);
                st_any |= 2;
                break;
              }
              const int stt = gdn_item(P, run, sm, B, bi, rec, conv, bm, s, L, i, w_in, r,
                                       spec ? sm.lmeta + nlog : nullptr,
                                       spec ? sm.lold + nlog : nullptr,
                                       (uint32_t)k << 10 | (uint32_t)(L - lo) << 12);
              if (spec && stt != ITEM_UNTOUCHED) nlog += bi.n_eager;
              if (stt == ITEM_WROTE) st_any |= 1;
              if (stt >= ITEM_PENDING) {
                st_any |= 2;
                pend |= 1 << k;
              }
            }
          }
          stp++;
        }
        PROF(PR_GITEMS);
        if (st_any) {
          sL = L;
          outL = st_any & 1;
          if (t < C)
            atomicMin(cluster.map_shared_rank(&sm.gkey[gpar], t), 2 * L + ((st_any & 2) ? 0 : 1));
          break;
        }
      }
      cluster.sync();
      COUNT(PR_BARRIERS);
      PROF(PR_GSYNC);
      const int key = *reinterpret_cast<volatile int*>(&sm.gkey[gpar]);
      gp++;
      if (key == 0x7fffffff) {  // every layer of the step done, none wrote
        lo = qhi;
        resume = false;
        rs_mask = 0;
        held_out = 0;
        continue;
      }
      const int J = key >> 1;
      for (int e = t; e < nlog; e += NT) {  // undo: the layers after J, J's pending items
        const uint32_t m = sm.lmeta[e];
        if (m == LXB_NOLOG) continue;
        const int lay = lo + (int)(m >> 12), kk = (int)(m >> 10) & 3;
        if (lay > J || (lay == J && sL == J && ((pend >> kk) & 1))) sm.win[m & 1023u] = sm.lold[e];
      }
      __syncthreads();
      if (!(key & 1)) {  // J has pending items: J again first, with only those
        resume = true;
        rs_mask = sL == J ? pend : 0;
        held_out = sL == J && outL;
        lo = J;
      } else {  // J wrote: its out_proj rows into the residual, then on from J + 1
        COUNT(PR_FIXUPS);
        ph++;
        const lxb_layer& lyJ = sm.layers[J];
        const lxb_owner ow = P.owners[lyJ.owner0 + rank];
        out_owner(P, sm, J, ow, rank, i, sm.own[ph & 1], cluster);
        __syncthreads();
        push_rows(P, sm, sm.own[ph & 1], ph & 1, rank * P.blk, P.blk, cluster);
        cluster.sync();
        COUNT(PR_BARRIERS);
        r_x = take_rows_norm(P, sm, ph & 1);
        x_new = false;
        ph++;
        PROF(PR_GFIXUP);
        resume = false;
        rs_mask = 0;
        held_out = 0;
        lo = J + 1;
      }
    }
    restage(hi);  // the step after the run: the next layer's blob (or the head's)
  };
  load_embed(run, P, sm, sm.tok);
  for (int i = 0; i < run.n_tokens; i++) {
    cur_tok = i;
    if (rank == 0 && t == 0 && run.inputs) run.inputs[(size_t)s * run.n_tokens + i] = sm.tok;
    for (int L = 0; L < P.n_layers;) {
      const lxb_layer& ly = sm.layers[L];
#if LXB_GROUPS
      // a run of GDN-only layers as group steps, except the layers whose items are all too big
      // to be speculated (each group step would take one of them, plus the pass's overhead)
      const unsigned long long big = sm.bigm;
      if (P.nbuf == 2 && ly.has_gdn && !ly.has_mlp && L + 1 < P.n_layers &&
          sm.layers[L + 1].has_gdn && !sm.layers[L + 1].has_mlp && !((big >> L) & 3ull)) {
        int hi = L + 1;
        while (hi < P.n_layers && sm.layers[hi].has_gdn && !sm.layers[hi].has_mlp &&
               !((big >> hi) & 1ull))
          hi++;
        group_run(L, hi, i);
        L = hi;
        continue;
      }
#endif
      cur_layer = L;
      const unsigned char* B = take(i);
      PROF(PR_WAIT);
      const lxb_bhdr bh = B ? *reinterpret_cast<const lxb_bhdr*>(B) : lxb_bhdr{};
      float* rec = reinterpret_cast<float*>(sm.sptr[L][0]);
      uint16_t* conv = reinterpret_cast<uint16_t*>(sm.sptr[L][1]);
      uint32_t* bm = run.bitmaps + ((size_t)s * P.n_layers + L) * LXB_NV * 8;
      if (x_new) {  // the norm factor changes with the residual only
        r_x = norm_factor(P, block_ssq(sm, sm.x));
        x_new = false;
      }
      const float r = r_x;
      const uint16_t* w_in = (B && bh.ln_in >= 0) ? reinterpret_cast<const uint16_t*>(B + bh.ln_in)
                                                 : P.u16 + ly.ln_in;
      const uint16_t* w_post = (B && bh.ln_post >= 0)
                                   ? reinterpret_cast<const uint16_t*>(B + bh.ln_post)
                                   : P.u16 + ly.ln_post;
      const bool mlp = ly.has_mlp && B && bh.mlp >= 0;
      lxb_bmlp mh{};
      if (mlp) mh = *reinterpret_cast<const lxb_bmlp*>(B + bh.mlp);
      int mr0 = mh.r0, mnr = mh.nr;  // this CTA's MLP rows
      if (ly.has_mlp && !mlp) {      // (no staged tables: the rows stay as they are)
        const lxb_owner o = P.owners[ly.owner0 + rank];
        mr0 = o.mr0;
        mnr = o.mr1 - o.mr0;
      }
      if (ly.has_gdn) {
        // this step's GDN input row into the ring (each CTA its block, 8 rows a thread of the
        // last two warps, which have the least to do at a step's start; rank 0 the factor)
        const size_t slot = ((size_t)s * P.n_layers + L) * 4 + (i & 3);
        uint4* rg = reinterpret_cast<uint4*>(run.ring + slot * H + rank * P.blk);
        for (int k = t - (NT - 64); k >= 0 && k < P.blk / 8; k += 64) {
          const float* xv = sm.x + rank * P.blk + 8 * k;
          rg[k] = make_uint4((uint32_t)lx_rb(xv[0]) | ((uint32_t)lx_rb(xv[1]) << 16),
                             (uint32_t)lx_rb(xv[2]) | ((uint32_t)lx_rb(xv[3]) << 16),
                             (uint32_t)lx_rb(xv[4]) | ((uint32_t)lx_rb(xv[5]) << 16),
                             (uint32_t)lx_rb(xv[6]) | ((uint32_t)lx_rb(xv[7]) << 16));
        }
        if (rank == 0 && t == NT - 1) run.ring_r[slot] = r;
      }
      if (ly.has_mlp) {  // (a step without one needs no barrier here: nothing above is read
        norm_into(sm.xm, sm.x, w_post, r);  // by another thread before the items' own barriers)
        if (t == 0) sm.qbad = 0u;
        __syncthreads();
      }
      if (P.nbuf == 2) issue_next(stp);  // the next step's blob: its buffer was read a step ago
      PROF(PR_NORM);
      // with an MLP the items are checked on its way and only the others run after it (they are
      // independent: the items read x, the MLP xm, and neither changes x before the barrier)
      // a layer whose GDN wrote at the last token most likely writes again (the real circuit's
      // first layers write at every token): its MLP runs once, after the out_proj rows, instead
      // of beside the items and again after them (the same in every CTA: the flags are)
      const bool unpair = ly.has_gdn && ly.has_mlp && B && ((sm.upm >> L) & 1ull);
      const bool merged = ly.has_gdn && B && mlp && !unpair;
      uint32_t todo = ly.has_gdn && B && !merged ? 0xffffffffu : 0u;  // items for gdn_item
      if (ly.has_mlp && !unpair) {
        if (mlp) todo |= mlp_owner(P, sm, B, mh, sm.own[ph & 1], merged ? w_in : nullptr, r);
        else copy_owner(sm, mr0, mnr, sm.own[ph & 1]);
        __syncthreads();
        push_rows(P, sm, sm.own[ph & 1], ph & 1, mr0, mnr, cluster);
      }
      PROF(PR_MLP);
      bool wrote = false;
      if (ly.has_gdn && B && todo) {
        const lxb_bhdr* bhp = reinterpret_cast<const lxb_bhdr*>(B);  // (dynamic index: in smem)
        for (int k = 0; k < bh.n_items; k++) {
          if (!((todo >> k) & 1)) continue;
          const lxb_bitem bi = *reinterpret_cast<const lxb_bitem*>(B + bhp->item[k]);
          wrote |= gdn_item(P, run, sm, B, bi, rec, conv, bm, s, L, i, w_in, r, nullptr, nullptr,
                            0) == ITEM_WROTE;
        }
      }
      if (wrote && t < C) *cluster.map_shared_rank(&sm.wflag[ph & 1], t) = 1;
      PROF(PR_ITEMS);
      cluster.sync();
      COUNT(PR_BARRIERS);
      PROF(PR_SYNC);
      const int fl = *reinterpret_cast<volatile int*>(&sm.wflag[ph & 1]);
      __syncthreads();
      if (t == 0 && ly.has_gdn && ly.has_mlp)  // (read at this layer's next step, many barriers on)
        sm.upm = fl ? sm.upm | 1ull << L : sm.upm & ~(1ull << L);
      if (fl || unpair) {
        if (fl) {  // the out_proj rows into the residual
          COUNT(PR_FIXUPS);
          if (t == 0) sm.wflag[ph & 1] = 0;
          if (P.nbuf == 1 && !ly.has_mlp) issue_next(stp);  // the blob is no longer read
          ph++;
          const lxb_owner ow = P.owners[ly.owner0 + rank];
          out_owner(P, sm, L, ow, rank, i, sm.own[ph & 1], cluster);
          __syncthreads();
          PROF(PR_FXOUT);
          push_rows(P, sm, sm.own[ph & 1], ph & 1, rank * P.blk, P.blk, cluster);
          cluster.sync();
          COUNT(PR_BARRIERS);
          r_x = take_rows_norm(P, sm, ph & 1);
          x_new = false;
          ph++;
          PROF(PR_FIXUP);
        }
        if (ly.has_mlp) {  // the MLP (again, or, unpaired and nothing written, now)
          if (fl) {
            norm_into(sm.xm, sm.x, w_post, r_x);
            __syncthreads();
          }
          if (mlp) mlp_owner(P, sm, B, mh, sm.own[ph & 1]);
          else copy_owner(sm, mr0, mnr, sm.own[ph & 1]);
          __syncthreads();
          push_rows(P, sm, sm.own[ph & 1], ph & 1, mr0, mnr, cluster);
          cluster.sync();
          COUNT(PR_BARRIERS);
          if (P.nbuf == 1) issue_next(stp);
          r_x = take_rows_norm(P, sm, ph & 1, ly.mrow0, ly.mrow1);
          ph++;
        }
        PROF(PR_FXMLP);
      } else {
        if (P.nbuf == 1) issue_next(stp);
        if (ly.has_mlp) r_x = take_rows_norm(P, sm, ph & 1, ly.mrow0, ly.mrow1);
        ph++;
        PROF(PR_PULL);
      }
      stp++;
      L++;
    }
    // the output head: every CTA its rows, then the first maximum over the cluster
    {
      cur_layer = P.n_layers;
      const unsigned char* B = take(i);
      PROF(PR_WAIT);
      const lxb_bhdr bh = B ? *reinterpret_cast<const lxb_bhdr*>(B) : lxb_bhdr{};
      if (x_new) {
        r_x = norm_factor(P, block_ssq(sm, sm.x));
        x_new = false;
      }
      const float r = r_x;
      norm_into(sm.xm, sm.x,
                B ? reinterpret_cast<const uint16_t*>(B + bh.ln_in) : P.u16 + P.final_norm, r);
      __syncthreads();
      // with helper clusters, rank 0 publishes the head input for them first
      const bool helped = run.n_help > 0 && !sm.help_dead;  // the same in every CTA
      const unsigned long long want = run.epoch | (unsigned long long)(i + 1);
      if (helped && rank == 0) {
        for (int k = t; k < H / 4; k += NT)
          reinterpret_cast<float4*>(run.hx)[k] = reinterpret_cast<const float4*>(sm.xm)[k];
        __syncthreads();
        if (t == 0) {
          __threadfence();
          st_release_u64(run.hseq, want);
        }
      }
      issue_next(stp);
      stp++;
      const int hsp = head_tables(P, sm);
      {  // this rank's first slices (helped), or its whole range
        float bv = -LXB_INF;
        int bi = 0x7fffffff;
        if (helped) {
          for (int k = 0; k < LXB_HEADMAIN; k++)
            head_rows(P, sm, P.headcta[rank * LXB_HEADSLICES + k], hsp, bv, bi);
        } else {
          head_rows(P, sm, P.headcta[C * LXB_HEADSLICES + rank], hsp, bv, bi);
        }
        head_reduce(sm, bv, bi);
      }
      cluster.sync();
      COUNT(PR_BARRIERS);
      cluster_max(sm, cluster, C);  // sm.cv / sm.ci: the cluster's first maximum
      if (helped) {
        // rank 0 gathers the helpers' maxima (each wait bounded) and tells every CTA
        if (rank == 0) {
          float hv = -LXB_INF;
          int hi = 0x7fffffff, ok = 1;
          if (t < run.n_help * C) {
            const uint4* hp = run.hpart + C + t;
            const long long t0 = clock64();
            for (;;) {
              uint32_t z;
              asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(z) : "l"(&hp->z) : "memory");
              if (z == (uint32_t)want && __ldcg(&hp->w) == (uint32_t)(want >> 32)) break;
              if (clock64() - t0 > (1ll << 26)) {  // ~34 ms: a helper is not there
                ok = 0;
                break;
              }
            }
            if (ok) {
              hv = __uint_as_float(__ldcg(&hp->x));
              hi = (int)__ldcg(&hp->y);
            }
          }
          if (t == 0 && (sm.cv > hv || (sm.cv == hv && sm.ci < hi))) {  // and the cluster's own
            hv = sm.cv;
            hi = sm.ci;
          }
          const int all = __syncthreads_and(ok);
          head_reduce(sm, hv, hi, &sm.gv, &sm.gi);  // not bestv: other CTAs may still read it
          if (t < C) {
            *cluster.map_shared_rank(&sm.hv, t) = sm.gv;
            *cluster.map_shared_rank(&sm.hi, t) = sm.gi;
            *cluster.map_shared_rank(&sm.hok, t) = all;
          }
        }
        cluster.sync();
        COUNT(PR_BARRIERS);
        if (sm.hok) {
          if (t == 0) {
            sm.cv = sm.hv;
            sm.ci = sm.hi;
          }
        } else {  // a helper is missing: the helpers' slices here, now and from now on
          float bv = sm.cv;
          int bi = sm.ci;
          __syncthreads();
          if (t == 0) sm.help_dead = 1;
          float v2 = -LXB_INF;
          int i2 = 0x7fffffff;
          for (int k = LXB_HEADMAIN; k < LXB_HEADSLICES; k++)
            head_rows(P, sm, P.headcta[rank * LXB_HEADSLICES + k], hsp, v2, i2);
          head_reduce(sm, v2, i2);
          cluster.sync();
          COUNT(PR_BARRIERS);
          cluster_max(sm, cluster, C);
          if (t == 0) {
            if (bv > sm.cv || (bv == sm.cv && bi < sm.ci)) {
              sm.cv = bv;
              sm.ci = bi;
            }
            if (rank == 0) {
              atomicOr(P.status, LXB_S_HELPER);
              st_release_u64(run.hseq, run.epoch | 0xffffffffull);  // the helpers may leave
            }
          }
        }
        __syncthreads();
      }
      {
        const int bi = sm.ci;  // the token: the first maximum of the logits
        if (t == 0) {
          if (rank == 0) run.preds[(size_t)s * run.n_tokens + i] = bi;
          int nt = (i + 1 < run.n_forced) ? run.forced[(size_t)s * run.n_forced + i + 1]
                                          : (run.typing.keys ? type_next(run, sm, s, bi) : bi);
          if (nt < 0 || (int64_t)nt + P.offset >= P.n_embed_rows) {
            if (i + 1 < run.n_tokens) set_status(P, LXB_S_TOKEN, s, i + 1);
            nt = 0;
          }
          // the next input enters the RX FIFO count when it is embedded in this launch; the
          // one after the last step is the next launch's first input and is counted there
          if (run.typing.keys && i + 1 < run.n_tokens) type_count(run, sm, nt);
          sm.tok = nt;
        }
      }
      __syncthreads();
      PROF(PR_HEAD);
      if (i + 1 < run.n_tokens) load_embed(run, P, sm, sm.tok);
      x_new = true;
      PROF(PR_EMBED);
      COUNT(PR_TOKENS);
    }
  }
#undef PROF
#undef COUNT
  if (prof && t == 0) {
    unsigned long long* d = run.prof + ((size_t)s * C + rank) * PR_N;
    for (int k = 0; k < PR_N; k++) d[k] += sm.pcs[k];
  }
  for (int k = t; k < sm.nwin; k += NT) {  // the resident conv windows back into the state
    const int L = P.winmap[2 * (sm.win0 + k)], ch = P.winmap[2 * (sm.win0 + k) + 1];
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(sm.sptr[L][1]) + (size_t)ch * 4) =
        sm.win[k];
  }
  if (run.n_help > 0 && rank == 0 && t == 0)  // a helper still waiting for a token may leave
    st_release_u64(run.hseq, run.epoch | 0xffffffffull);
  if (run.typing.keys && rank == 0 && t == 0) {  // the queue's state, and the next input
    int32_t* ts = run.typing.tstate + (size_t)s * 4;
    ts[0] = sm.tq_k;
    ts[1] = sm.tq_wait;
    ts[2] = sm.tq_left;
    ts[3] = sm.tok;
  }
  cluster.sync();  // every ring write of the launch is visible cluster-wide
  materialize(P, run, sm, s, rank, run.n_tokens);
  cluster.sync();  // no CTA leaves while another may still read its shared memory
}

// the nonzero-row bitmaps of the decaying layers' states: one warp per state row
__global__ void lxb_bitmap_kernel(const uint64_t* state_ptrs, uint32_t* bitmaps,
                                  const lxb_layer* layers, int n_layers) {
  const int s = blockIdx.z, L = blockIdx.y, vh = blockIdx.x;
  if (!layers[L].decays) return;
  const float* S = reinterpret_cast<const float*>(state_ptrs[((size_t)s * n_layers + L) * 2]) +
                   (size_t)vh * KD * VD;
  uint32_t* b = bitmaps + (((size_t)s * n_layers + L) * LXB_NV + vh) * 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;  // 8 warps
  for (int w = warp; w < 8; w += 8) {
    uint32_t word = 0;
    for (int i = 0; i < 32; i++) {
      const float4 v = reinterpret_cast<const float4*>(S + (size_t)(w * 32 + i) * VD)[lane];
      const bool nz = v.x != 0.0f || v.y != 0.0f || v.z != 0.0f || v.w != 0.0f;
      if (__any_sync(0xffffffffu, nz)) word |= 1u << i;
    }
    if (lane == 0) b[w] = word;
  }
}

// =============================================================================================
// The C ABI
// =============================================================================================
struct lxb_plan {
  int device;
  int cluster;
  void* dimage;
  size_t bytes;
  lxb_image_header hdr;
  Dev dev;
  uint32_t* status;
  int max_clusters;
  int head_helpers;              // the most head helper clusters a single-stream launch may use
  int help_drill;                // helpers that never answer (lxb_plan_set_head_helpers < 0)
  unsigned long long* prof;
  int smem;  // dynamic shared memory per CTA: Smem, then the staging buffers
  lxb_typing typing;             // the device typing queue (keys == null: off)
};

static_assert(offsetof(Smem, own) % 16 == 0 && offsetof(Smem, on) % 16 == 0 && offsetof(Smem, xin) % 16 == 0 &&
                  offsetof(Smem, onall) % 16 == 0 && offsetof(Smem, mbar) % 8 == 0 &&
                  sizeof(Smem) < 160 * 1024,
              "shared memory layout");

static int cuda_rc(cudaError_t e) { return e == cudaSuccess ? LXB_OK : (int)e; }

extern "C" int lxb_abi_version(void) { return LXB_ABI_VERSION; }

extern "C" int lxb_query(int device, lxb_caps* caps) {
  if (!caps) return LXB_E_INVAL;
  memset(caps, 0, sizeof(*caps));
  caps->device = device;
  cudaError_t e;
  if ((e = cudaDeviceGetAttribute(&caps->cc_major, cudaDevAttrComputeCapabilityMajor, device)))
    return cuda_rc(e);
  cudaDeviceGetAttribute(&caps->cc_minor, cudaDevAttrComputeCapabilityMinor, device);
  cudaDeviceGetAttribute(&caps->sm_count, cudaDevAttrMultiProcessorCount, device);
  cudaDeviceGetAttribute(&caps->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  cudaDeviceGetAttribute(&caps->cluster_launch, cudaDevAttrClusterLaunch, device);
  return LXB_OK;
}

const char* lxb_error_string_c(int code) {
  switch (code) {
    case LXB_OK: return "ok";
    case LXB_E_INVAL: return "invalid argument";
    case LXB_E_IMAGE: return "malformed plan image";
    case LXB_E_DEVICE: return "device cannot run this plan";
    case LXB_E_STATUS: return "kernel reported an error (lxb_status)";
    case LXB_E_TOOBIG:
      return "the request needs more scratch than lxb_decode_noalloc's fixed array holds";
    default: return code > 0 ? cudaGetErrorString((cudaError_t)code) : "unknown error";
  }
}
extern "C" const char* lxb_error_string(int code) { return lxb_error_string_c(code); }

// --- image validation: every offset, count and index the kernel will follow ------------------
namespace {
struct View {
  const unsigned char* base;
  size_t bytes;
  const lxb_image_header* h;
  template <class T>
  const T* sec(int k) const { return reinterpret_cast<const T*>(base + h->sec[k].off); }
  int64_t n(int k) const { return h->sec[k].count; }
};

bool ent_range(const View& v, int64_t off, int64_t cnt) {
  return off >= 0 && cnt >= 0 && off + cnt <= v.n(LXB_SEC_ENT);
}
bool i32_range(const View& v, int64_t off, int64_t cnt) {
  return off >= 0 && cnt >= 0 && off + cnt <= v.n(LXB_SEC_I32);
}
bool u16_range(const View& v, int64_t off, int64_t cnt) {
  return off >= 0 && cnt >= 0 && off + cnt <= v.n(LXB_SEC_U16);
}
// entries [off, off + cnt) whose low 16 bits must be < lim
bool ent_idx(const View& v, int64_t off, int64_t cnt, uint32_t lim) {
  if (!ent_range(v, off, cnt)) return false;
  const uint32_t* e = v.sec<uint32_t>(LXB_SEC_ENT) + off;
  for (int64_t i = 0; i < cnt; i++)
    if ((e[i] & 0xffffu) >= lim) return false;
  return true;
}
// a row-pointer block: n + 1 monotone pointers into ent, entries' indices < lim
bool rowptr_ok(const View& v, int32_t p, int n, uint32_t lim) {
  if (!i32_range(v, p, (int64_t)n + 1)) return false;
  const int32_t* rp = v.sec<int32_t>(LXB_SEC_I32) + p;
  for (int k = 0; k < n; k++)
    if (rp[k + 1] < rp[k]) return false;
  return ent_idx(v, rp[0], (int64_t)rp[n] - rp[0], lim);
}

// the step blobs: every offset, count and index the kernel follows inside one
bool blob_rng(int64_t off, int64_t len, int64_t bytes, int align = 4) {
  return off >= 0 && len >= 0 && off % align == 0 && off + len <= bytes;
}
bool blob_ent(const unsigned char* B, int64_t bytes, int64_t off, int64_t n, uint32_t lim) {
  if (!blob_rng(off, 4 * n, bytes)) return false;
  const uint32_t* e = reinterpret_cast<const uint32_t*>(B + off);
  for (int64_t i = 0; i < n; i++)
    if ((e[i] & 0xffffu) >= lim) return false;
  return true;
}

int validate_blobs(const View& v, int C) {
  const lxb_image_header* h = v.h;
  const int nl = h->n_layers;
  if (v.n(LXB_SEC_BLOBIDX) != (int64_t)(nl + 1) * C || h->blob_max < (int)sizeof(lxb_bhdr) ||
      h->blob_max % 16)
    return LXB_E_IMAGE;
  const lxb_blobref* refs = v.sec<lxb_blobref>(LXB_SEC_BLOBIDX);
  const unsigned char* base = v.sec<unsigned char>(LXB_SEC_BLOBS);
  const lxb_layer* layers = v.sec<lxb_layer>(LXB_SEC_LAYERS);
  const lxb_item* items = v.sec<lxb_item>(LXB_SEC_ITEMS);
  const lxb_chan* gchans = v.sec<lxb_chan>(LXB_SEC_CHANS);
  const uint32_t* gent = v.sec<uint32_t>(LXB_SEC_ENT);
  if (v.n(LXB_SEC_WINIDX) != C) return LXB_E_IMAGE;
  const int32_t* widx = v.sec<int32_t>(LXB_SEC_WINIDX);
  const int32_t* wmap = v.sec<int32_t>(LXB_SEC_WINMAP);
  for (int c = 0; c < C; c++)
    if (widx[2 * c] < 0 || widx[2 * c + 1] < 0 || widx[2 * c + 1] > LXB_MAXWIN ||
        (int64_t)widx[2 * c] + widx[2 * c + 1] > v.n(LXB_SEC_WINMAP))
      return LXB_E_IMAGE;
  for (int64_t k = 0; k < v.n(LXB_SEC_WINMAP); k++)
    if (wmap[2 * k] < 0 || wmap[2 * k] >= nl || wmap[2 * k + 1] < 0 ||
        wmap[2 * k + 1] >= LXB_CONV)
      return LXB_E_IMAGE;
  for (int L = 0; L <= nl; L++) {
    for (int c = 0; c < C; c++) {
      const lxb_blobref& br = refs[L * C + c];
      if (br.off < 0 || br.off % 16 || br.bytes < (int)sizeof(lxb_bhdr) || br.bytes % 16 ||
          br.bytes > h->blob_max || br.off + br.bytes > v.n(LXB_SEC_BLOBS))
        return LXB_E_IMAGE;
      const unsigned char* B = base + br.off;
      const int64_t nb = br.bytes;
      const lxb_bhdr* bh = reinterpret_cast<const lxb_bhdr*>(B);
      if (bh->bytes != br.bytes) return LXB_E_IMAGE;
      if (L == nl) {  // the head's blob: the final norm
        if (!blob_rng(bh->ln_in, 2 * H, nb, 16)) return LXB_E_IMAGE;
        continue;
      }
      const lxb_layer& ly = layers[L];
      if (ly.has_gdn && !blob_rng(bh->ln_in, 2 * H, nb, 16)) return LXB_E_IMAGE;
      if (ly.has_mlp && !blob_rng(bh->ln_post, 2 * H, nb, 16)) return LXB_E_IMAGE;
      if (bh->n_items < 0 || bh->n_items > LXB_ITEMSLOTS || (bh->n_items && !ly.has_gdn))
        return LXB_E_IMAGE;
      for (int k = 0; k < bh->n_items; k++) {
        if (!blob_rng(bh->item[k], sizeof(lxb_bitem), nb, 16)) return LXB_E_IMAGE;
        const lxb_bitem& bi = *reinterpret_cast<const lxb_bitem*>(B + bh->item[k]);
        if (bi.item < ly.item0 || bi.item >= ly.item0 + ly.n_items) return LXB_E_IMAGE;
        const lxb_item& it = items[bi.item];
        if (it.cta != c || it.kh != bi.kh || it.slot != bi.slot || it.flags != bi.flags ||
            bi.n_eager != it.n_eager || bi.n_eager < 0 || bi.n_eager > 2 * LXB_KD ||
            bi.n_eager > it.n_ch)
          return LXB_E_IMAGE;
        if (!blob_rng(bi.eager, (int64_t)bi.n_eager * sizeof(lxb_bchan), nb, 16))
          return LXB_E_IMAGE;
        for (int e = 0; e < bi.n_eager; e++) {
          const lxb_bchan& ch = reinterpret_cast<const lxb_bchan*>(B + bi.eager)[e];
          if (ch.slot >= 2 * LXB_KD || ch.conv_ch >= LXB_CONV || !blob_ent(B, nb, ch.ent, ch.n, H))
            return LXB_E_IMAGE;
          if (ch.win == LXB_NOWIN && !(bi.flags & LXB_IT_NONRES)) return LXB_E_IMAGE;
          // the global table's record of the channel (the quiet pass reads that one): the same
          // window, taps and entries
          const lxb_chan& gc = gchans[it.ch0 + e];
          if (gc.win != ch.win || gc.n != ch.n || gc.conv_ch != ch.conv_ch || gc.t01 != ch.t01 ||
              gc.t23 != ch.t23)
            return LXB_E_IMAGE;
          for (int q = 0; q < ch.n; q++)
            if (gent[gc.ent + q] != reinterpret_cast<const uint32_t*>(B + ch.ent)[q])
              return LXB_E_IMAGE;
          if (ch.win != LXB_NOWIN) {  // a resident window: the map must name this channel
            if (ch.win >= (uint32_t)widx[2 * c + 1]) return LXB_E_IMAGE;
            const int32_t* wp = wmap + 2 * ((int64_t)widx[2 * c] + ch.win);
            if (wp[0] != L || wp[1] != (int32_t)ch.conv_ch) return LXB_E_IMAGE;
          }
        }
        if (!blob_rng(bi.rows, 16 * 8, nb, 16) || !blob_rng(bi.prm, 2 * (2 * R + VD), nb, 16))
          return LXB_E_IMAGE;
        const int32_t* rr = reinterpret_cast<const int32_t*>(B + bi.rows);
        for (int q = 0; q < 2 * R; q++)
          if (!blob_ent(B, nb, rr[2 * q], rr[2 * q + 1], H)) return LXB_E_IMAGE;
        if (bi.z >= 0) {  // the in_proj_z rows: 1025 pointers, then the entries
          if (!blob_rng(bi.z, 4 * 1025, nb, 16)) return LXB_E_IMAGE;
          const int32_t* zp = reinterpret_cast<const int32_t*>(B + bi.z);
          if (zp[0] != 0) return LXB_E_IMAGE;
          for (int k = 0; k < 1024; k++)
            if (zp[k + 1] < zp[k]) return LXB_E_IMAGE;
          if (!blob_ent(B, nb, bi.z + ((4 * 1025 + 15) & ~15), zp[1024], H)) return LXB_E_IMAGE;
        } else if (bi.flags & LXB_IT_OUT) {
          return LXB_E_IMAGE;  // a head that can write needs its z rows
        }
      }
      if (ly.has_mlp) {
        if (!blob_rng(bh->mlp, sizeof(lxb_bmlp), nb, 16)) return LXB_E_IMAGE;
        const lxb_bmlp& m = *reinterpret_cast<const lxb_bmlp*>(B + bh->mlp);
        const lxb_owner& ow = v.sec<lxb_owner>(LXB_SEC_OWNERS)[L * C + c];  // (checked)
        if (m.n_units < 0 || m.n_units > LXB_MAXUNITS || m.r0 != ow.mr0 ||
            m.nr != ow.mr1 - ow.mr0 ||
            !blob_rng(m.units, (int64_t)m.n_units * sizeof(lxb_bunit), nb, 16) ||
            !blob_rng(m.down_ptr, 4 * (int64_t)(m.nr + 1), nb, 16))
          return LXB_E_IMAGE;
        const lxb_bunit* un = reinterpret_cast<const lxb_bunit*>(B + m.units);
        for (int u = 0; u < m.n_units; u++)
          if (!blob_ent(B, nb, un[u].g, un[u].ng, H) || !blob_ent(B, nb, un[u].u, un[u].nu, H))
            return LXB_E_IMAGE;
        if (m.n_units) {  // the kernel indexes the units' products from the first gate entry
          const int64_t g0 = un[0].g, end = un[m.n_units - 1].u + 4 * (int64_t)un[m.n_units - 1].nu;
          for (int u = 0; u < m.n_units; u++)
            if (un[u].g < g0 || un[u].g + 4 * (int64_t)un[u].ng > end || un[u].u < g0 ||
                un[u].u + 4 * (int64_t)un[u].nu > end)
              return LXB_E_IMAGE;
        }
        const int32_t* rp = reinterpret_cast<const int32_t*>(B + m.down_ptr);
        if (rp[0] != 0) return LXB_E_IMAGE;
        for (int k = 0; k < m.nr; k++)
          if (rp[k + 1] < rp[k]) return LXB_E_IMAGE;
        if (!blob_ent(B, nb, m.down_ent, rp[m.nr], (uint32_t)m.n_units)) return LXB_E_IMAGE;
      }
    }
  }
  return LXB_OK;
}

int validate(const View& v, int cluster) {
  const lxb_image_header* h = v.h;
  if (v.bytes < sizeof(lxb_image_header)) return LXB_E_IMAGE;
  if (h->magic != LXB_MAGIC || h->version != LXB_IMAGE_VERSION) return LXB_E_IMAGE;
  if (h->hidden != H || h->cluster != cluster || h->n_layers < 1 ||
      h->n_layers > LXB_MAXLAYERS || h->n_vocab < 1)
    return LXB_E_IMAGE;
  const size_t esz[LXB_SEC_COUNT] = {sizeof(lxb_layer), sizeof(lxb_item), sizeof(lxb_chan), 4,
                                     sizeof(lxb_unit), sizeof(lxb_owner), 4, 2,
                                     sizeof(lxb_headcta), 8, 1, sizeof(lxb_blobref), 8, 8};
  for (int k = 0; k < LXB_SEC_COUNT; k++) {
    const lxb_sec& s = h->sec[k];
    if (s.off < (int64_t)sizeof(lxb_image_header) || s.off % 16 || s.count < 0 ||
        (size_t)s.off + (size_t)s.count * esz[k] > v.bytes)
      return LXB_E_IMAGE;
  }
  const int C = cluster, blk = H / C;
  if (v.n(LXB_SEC_LAYERS) != h->n_layers || v.n(LXB_SEC_OWNERS) != (int64_t)h->n_layers * C ||
      v.n(LXB_SEC_HEADCTA) != (int64_t)C * (LXB_HEADSLICES + 1) || v.n(LXB_SEC_ITEMS) != h->n_items)
    return LXB_E_IMAGE;
  if (h->n_dense < 0 || h->n_dense > LXB_MAXDENSE) return LXB_E_IMAGE;
  if (h->n_dense && v.n(LXB_SEC_HCODES) != h->n_vocab) return LXB_E_IMAGE;
  for (int j = 0; j < h->n_dense; j++)
    if (h->dense_cols[j] < 0 || h->dense_cols[j] >= H) return LXB_E_IMAGE;
  if (!u16_range(v, h->final_norm, H) || h->n_embed_rows < 1 || h->offset < 0) return LXB_E_IMAGE;
  if (h->hsp_mask != -1 && !i32_range(v, h->hsp_mask, H / 32)) return LXB_E_IMAGE;
  const lxb_layer* layers = v.sec<lxb_layer>(LXB_SEC_LAYERS);
  const lxb_item* items = v.sec<lxb_item>(LXB_SEC_ITEMS);
  const lxb_chan* chans = v.sec<lxb_chan>(LXB_SEC_CHANS);
  const lxb_owner* owners = v.sec<lxb_owner>(LXB_SEC_OWNERS);
  for (int L = 0; L < h->n_layers; L++) {
    const lxb_layer& ly = layers[L];
    if (!u16_range(v, ly.ln_in, H) || !u16_range(v, ly.ln_post, H)) return LXB_E_IMAGE;
    if (ly.item0 < 0 || ly.n_items < 0 || ly.item0 + ly.n_items > h->n_items) return LXB_E_IMAGE;
    if (ly.owner0 != L * C) return LXB_E_IMAGE;
    if (!i32_range(v, ly.itemof, LXB_NK)) return LXB_E_IMAGE;
    const int32_t* io = v.sec<int32_t>(LXB_SEC_I32) + ly.itemof;
    for (int kh = 0; kh < LXB_NK; kh++)
      if (io[kh] != -1 && (io[kh] < ly.item0 || io[kh] >= ly.item0 + ly.n_items ||
                           items[io[kh]].kh != kh))
        return LXB_E_IMAGE;
    int per_cta[LXB_MAXC] = {0};
    for (int k = 0; k < ly.n_items; k++) {
      const lxb_item& it = items[ly.item0 + k];
      if (it.layer != L || it.kh < 0 || it.kh >= LXB_NK || it.cta < 0 || it.cta >= C ||
          it.slot < 0 || it.slot >= LXB_ITEMSLOTS || io[it.kh] != ly.item0 + k)
        return LXB_E_IMAGE;
      if (per_cta[it.cta] & (1 << it.slot)) return LXB_E_IMAGE;  // one item per (cta, slot)
      per_cta[it.cta] |= 1 << it.slot;
      if (it.ch0 < 0 || it.n_ch < 0 || it.n_ch > LXB_NSLOT || it.n_eager < 0 ||
          it.n_vneed < 0 || it.n_eager + it.n_vneed > it.n_ch ||
          (int64_t)it.ch0 + it.n_ch > v.n(LXB_SEC_CHANS))
        return LXB_E_IMAGE;
      for (int c = 0; c < it.n_ch; c++) {
        const lxb_chan& ch = chans[it.ch0 + c];
        const bool computed = c < it.n_eager + it.n_vneed;  // these write their q|k|v slot
        if (ch.conv_ch >= LXB_CONV || ch.tapmask > 15 ||
            (computed ? ch.slot >= LXB_NSLOT : (ch.slot != LXB_NOSLOT && ch.slot >= LXB_NSLOT)) ||
            !ent_idx(v, ch.ent, ch.n, H))
          return LXB_E_IMAGE;
      }
      if (!i32_range(v, it.rows, 2 * (2 * R + R * VD)) || !u16_range(v, it.params, 2 * R + VD))
        return LXB_E_IMAGE;
      const int32_t* rr = v.sec<int32_t>(LXB_SEC_I32) + it.rows;
      for (int q = 0; q < 2 * R + R * VD; q++)
        if (!ent_idx(v, rr[2 * q], rr[2 * q + 1], H)) return LXB_E_IMAGE;
      if ((it.flags & LXB_IT_DECAYS) && !ly.decays) return LXB_E_IMAGE;
    }
    for (int c = 0; c < C; c++) {
      const lxb_owner& ow = owners[L * C + c];
      // the MLP row ranges: 8-row aligned, at most BLKMAX rows, tiling [mrow0, mrow1) in order
      if (ow.mr0 < 0 || ow.mr1 < ow.mr0 || ow.mr1 > H || (ow.mr0 & 7) || (ow.mr1 & 7) ||
          ow.mr1 - ow.mr0 > BLKMAX || ow.mr0 != (c ? owners[L * C + c - 1].mr1 : ly.mrow0) ||
          (c == C - 1 && ow.mr1 != ly.mrow1) || (!ly.has_mlp && ow.mr1 != ow.mr0))
        return LXB_E_IMAGE;
      if (ow.orow >= 0 && !rowptr_ok(v, ow.orow, blk, LXB_NV * LXB_VD)) return LXB_E_IMAGE;
    }
  }
  const lxb_headcta* hc = v.sec<lxb_headcta>(LXB_SEC_HEADCTA);
  int prev = 0;
  for (int c = 0; c < C * LXB_HEADSLICES; c++) {
    if (hc[c].r0 != prev || hc[c].r1 < hc[c].r0 || hc[c].r1 > h->n_vocab) return LXB_E_IMAGE;
    prev = hc[c].r1;
    if (!rowptr_ok(v, hc[c].rowptr, hc[c].r1 - hc[c].r0, H)) return LXB_E_IMAGE;
  }
  if (prev != h->n_vocab) return LXB_E_IMAGE;
  for (int c = 0; c < C; c++) {  // each rank's whole range: its slices together
    const lxb_headcta& w = hc[C * LXB_HEADSLICES + c];
    if (w.r0 != hc[c * LXB_HEADSLICES].r0 || w.r1 != hc[c * LXB_HEADSLICES + LXB_HEADSLICES - 1].r1)
      return LXB_E_IMAGE;
    if (!rowptr_ok(v, w.rowptr, w.r1 - w.r0, H)) return LXB_E_IMAGE;
  }
  if (h->n_dense) {
    const uint64_t* codes = v.sec<uint64_t>(LXB_SEC_HCODES);
    const int bits = 2 * h->n_dense;
    for (int64_t r = 0; r < h->n_vocab; r++)
      if (bits < 64 && (codes[r] >> bits)) return LXB_E_IMAGE;
  }
  return validate_blobs(v, cluster);
}
}  // namespace

extern "C" int lxb_plan_create(const void* image, size_t bytes, int cluster, lxb_plan** out) {
  if (!image || !out || bytes < sizeof(lxb_image_header)) return LXB_E_INVAL;
  *out = nullptr;
  if (cluster < LXB_MINC || cluster > LXB_MAXC || H % cluster || (H / cluster) % 4)
    return LXB_E_INVAL;
  View v{static_cast<const unsigned char*>(image), bytes,
         static_cast<const lxb_image_header*>(image)};
  int rc = validate(v, cluster);
  if (rc) return rc;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e) return cuda_rc(e);
  int major = 0, cl = 0, optin = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&cl, cudaDevAttrClusterLaunch, dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int base = (int)((sizeof(Smem) + 127) / 128 * 128);
  // two staging buffers; when the largest blob does not fit twice, buffers of what does fit,
  // and the larger blobs are read in global memory (stage_issue)
  int stage = (v.h->blob_max + 127) / 128 * 128;
  if (base + 2 * stage > optin) stage = (optin - base) / 2 / 128 * 128;
  const int nbuf = 2;
  if (major < 10 || !cl || stage < (int)sizeof(lxb_bhdr)) return LXB_E_DEVICE;
  lxb_plan* p = new (std::nothrow) lxb_plan();
  if (!p) return LXB_E_INVAL;
  p->device = dev;
  p->cluster = cluster;
  p->bytes = bytes;
  p->hdr = *v.h;
  if ((e = cudaMalloc(&p->dimage, bytes))) {
    delete p;
    return cuda_rc(e);
  }
  if ((e = cudaMalloc(&p->status, 16)) || (e = cudaMemset(p->status, 0, 16)) ||
      (e = cudaMemcpy(p->dimage, image, bytes, cudaMemcpyHostToDevice))) {
    cudaFree(p->dimage);
    if (p->status) cudaFree(p->status);
    delete p;
    return cuda_rc(e);
  }
  const unsigned char* b = static_cast<const unsigned char*>(p->dimage);
  const lxb_image_header* h = &p->hdr;
  Dev& d = p->dev;
  d.layers = reinterpret_cast<const lxb_layer*>(b + h->sec[LXB_SEC_LAYERS].off);
  d.items = reinterpret_cast<const lxb_item*>(b + h->sec[LXB_SEC_ITEMS].off);
  d.chans = reinterpret_cast<const lxb_chan*>(b + h->sec[LXB_SEC_CHANS].off);
  d.ent = reinterpret_cast<const uint32_t*>(b + h->sec[LXB_SEC_ENT].off);
  d.units = reinterpret_cast<const lxb_unit*>(b + h->sec[LXB_SEC_UNITS].off);
  d.owners = reinterpret_cast<const lxb_owner*>(b + h->sec[LXB_SEC_OWNERS].off);
  d.i32 = reinterpret_cast<const int32_t*>(b + h->sec[LXB_SEC_I32].off);
  d.u16 = reinterpret_cast<const uint16_t*>(b + h->sec[LXB_SEC_U16].off);
  d.headcta = reinterpret_cast<const lxb_headcta*>(b + h->sec[LXB_SEC_HEADCTA].off);
  d.hcodes = reinterpret_cast<const uint64_t*>(b + h->sec[LXB_SEC_HCODES].off);
  d.n_layers = h->n_layers;
  d.C = cluster;
  d.blk = H / cluster;
  d.n_vocab = h->n_vocab;
  d.n_dense = h->n_dense;
  d.final_norm = h->final_norm;
  d.eps = h->eps;
  d.n_embed_rows = h->n_embed_rows;
  d.offset = h->offset;
  memcpy(d.htab, h->htab, sizeof(d.htab));
  memcpy(d.dense_cols, h->dense_cols, sizeof(d.dense_cols));
  d.hsp = h->hsp_mask >= 0 ? reinterpret_cast<const uint32_t*>(d.i32 + h->hsp_mask) : nullptr;
  d.status = p->status;
  d.blobs = b + h->sec[LXB_SEC_BLOBS].off;
  d.blobidx = reinterpret_cast<const lxb_blobref*>(b + h->sec[LXB_SEC_BLOBIDX].off);
  d.winmap = reinterpret_cast<const int32_t*>(b + h->sec[LXB_SEC_WINMAP].off);
  d.winidx = reinterpret_cast<const int32_t*>(b + h->sec[LXB_SEC_WINIDX].off);
  d.nbuf = nbuf;
  d.stage = stage;
  p->smem = base + nbuf * stage;
  // launch attributes, and how many clusters fit at once
  const int smem = p->smem;
  cudaFuncSetAttribute(lxb_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (cluster > 8)
    cudaFuncSetAttribute(lxb_decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(cluster);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int ncl = 0;
  e = cudaOccupancyMaxActiveClusters(&ncl, (void*)lxb_decode_kernel, &cfg);
  if (e || ncl < 1) {
    cudaGetLastError();
    lxb_plan_destroy(p);
    return e ? cuda_rc(e) : LXB_E_DEVICE;
  }
  p->max_clusters = ncl;
  p->head_helpers = LXB_HEADSLICES - 1;
  p->help_drill = 0;
  *out = p;
  return LXB_OK;
}

static size_t ring_bytes(const lxb_plan* p, int n_streams) {
  return (size_t)n_streams * p->hdr.n_layers * 4 * H * sizeof(uint16_t);
}

// the head helpers' exchange, after the ring and its factors: hx [2560] float, hseq, hpart
static size_t head_xchg_bytes(const lxb_plan* p) {
  return (size_t)H * 4 + 16 + (size_t)p->cluster * LXB_HEADSLICES * 16;
}

extern "C" size_t lxb_scratch_bytes(const lxb_plan* p, int n_streams) {
  if (!p || n_streams < 1) return 0;
  const size_t base =
      ring_bytes(p, n_streams) + (size_t)n_streams * p->hdr.n_layers * 4 * sizeof(float);
  return ((base + 15) & ~(size_t)15) + head_xchg_bytes(p);
}

// the head helpers' launch epochs (see decode_launch)
static std::atomic<unsigned long long> g_launch_epoch{0};

static int decode_launch(lxb_plan* p, const uint64_t* state_ptrs, uint32_t* bitmaps,
                         int sync_bitmaps, void* scratch, const uint16_t* embed, int n_streams,
                         const int32_t* forced, int n_forced, int n_tokens, int32_t* preds,
                         int32_t* inputs, void* cuda_stream) {
  if (!p || !state_ptrs || !bitmaps || !scratch || !embed || !forced || !preds ||
      n_streams < 1 || n_forced < 1 || n_tokens < 1 || n_streams > 65535)
    return LXB_E_INVAL;
  if ((reinterpret_cast<uintptr_t>(embed) & 15) || (reinterpret_cast<uintptr_t>(bitmaps) & 15) ||
      (reinterpret_cast<uintptr_t>(scratch) & 15))
    return LXB_E_INVAL;
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  cudaError_t e;
  if (sync_bitmaps) {
    lxb_bitmap_kernel<<<dim3(LXB_NV, p->hdr.n_layers, n_streams), 256, 0, st>>>(
        state_ptrs, bitmaps, p->dev.layers, p->hdr.n_layers);
    if ((e = cudaGetLastError())) return cuda_rc(e);
  }
  uint16_t* ring = static_cast<uint16_t*>(scratch);
  float* ring_r = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) +
                                           ring_bytes(p, n_streams));
  unsigned char* xg =
      static_cast<unsigned char*>(scratch) +
      ((ring_bytes(p, n_streams) + (size_t)n_streams * p->hdr.n_layers * 4 * sizeof(float) + 15) &
       ~(size_t)15);
  // head helpers: a single stream, clusters the device can hold beside it, tokens the tag counts
  int n_help = 0;
  if (n_streams == 1 && n_tokens < 0x7fffffff)
    n_help = std::min(std::min(p->head_helpers, LXB_HEADSLICES - LXB_HEADMAIN), p->max_clusters - 1);
  if (n_help < 0) n_help = 0;
  // The helpers' exchange words are tagged (launch epoch | token + 1). The epoch comes from one
  // counter for the whole process, so no two launches share it, whichever plans they belong to;
  // and the words are cleared on the stream before the launch, so nothing another launch (or
  // another process) left in this scratch memory can match a tag: 0 is never a valid tag.
  const unsigned long long epoch = (g_launch_epoch.fetch_add(1) + 1) << 32;
  if (n_help > 0) {
    e = cudaMemsetAsync(xg + (size_t)H * 4, 0, head_xchg_bytes(p) - (size_t)H * 4, st);
    if (e) return cuda_rc(e);
  }
  Run run{state_ptrs, bitmaps, ring, ring_r, embed, forced, n_forced, n_tokens, preds, inputs,
          p->prof, n_streams, n_help, reinterpret_cast<float*>(xg),
          reinterpret_cast<unsigned long long*>(xg + (size_t)H * 4),
          reinterpret_cast<uint4*>(xg + (size_t)H * 4 + 16), epoch, p->help_drill, p->typing};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = p->cluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(p->cluster * (n_streams + n_help));
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = p->smem;
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, lxb_decode_kernel, p->dev, run);
  return cuda_rc(e);
}

extern "C" int lxb_decode(lxb_plan* p, const uint64_t* state_ptrs, uint32_t* bitmaps,
                          int sync_bitmaps, void* scratch, const uint16_t* embed, int n_streams,
                          const int32_t* forced, int n_forced, int n_tokens, int32_t* preds,
                          int32_t* inputs, void* cuda_stream) {
  return decode_launch(p, state_ptrs, bitmaps, sync_bitmaps, scratch, embed, n_streams, forced,
                       n_forced, n_tokens, preds, inputs, cuda_stream);
}

// --- decoding without allocating -------------------------------------------------------------
// Some hosts cannot give this library any device memory after start-up: a serving process whose
// device memory is one pool carved up when it starts, or a host whose allocator is not
// CUDA-aware and hands out only the buffers it manages (state, tokens, predictions). For them the
// decode's scratch (the 4-step residual ring of the lazily kept conv windows) lives in this
// file-scope device array instead of a caller buffer. Every GPU that loads the library holds it
// until the process exits. All calls on a device share it and it keeps the last call's contents.
// The kernel writes every ring slot before it reads it; the head helpers' exchange words, which
// must not match a tag from an earlier call, are cleared on the stream before every launch that
// uses helpers (decode_launch). Two calls that overlap on the GPU (other streams, other threads)
// race on the array.
static __device__ __align__(256) unsigned char lxb_noalloc_scratch[LXB_NOALLOC_MAX_SCRATCH];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[LXB_MAX_DEVICES];  // the array's device address, per device

extern "C" int lxb_decode_noalloc(lxb_plan* p, const uint64_t* state_ptrs, uint32_t* bitmaps,
                                  int sync_bitmaps, const uint16_t* embed, int n_streams,
                                  const int32_t* forced, int n_forced, int n_tokens,
                                  int32_t* preds, int32_t* inputs, void* cuda_stream) {
  if (!p || n_streams < 1) return LXB_E_INVAL;
  if (lxb_scratch_bytes(p, n_streams) > LXB_NOALLOC_MAX_SCRATCH) return LXB_E_TOOBIG;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e) return cuda_rc(e);
  if (dev != p->device || dev < 0 || dev >= LXB_MAX_DEVICES) return LXB_E_INVAL;
  void* ptr = nullptr;
  {
    // set-up, once per device, with that device current: the host-side name of the array is
    // not its device address
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      e = cudaGetSymbolAddress(&ptr, lxb_noalloc_scratch);
      if (e) return cuda_rc(e);
      g_noalloc_ptr[dev] = ptr;
    }
    ptr = g_noalloc_ptr[dev];
  }
  return decode_launch(p, state_ptrs, bitmaps, sync_bitmaps, ptr, embed, n_streams, forced,
                       n_forced, n_tokens, preds, inputs, cuda_stream);
}

extern "C" int lxb_status(lxb_plan* p, lxb_error* err) {
  if (!p || !err) return LXB_E_INVAL;
  uint32_t s[3];
  cudaError_t e = cudaMemcpy(s, p->status, 12, cudaMemcpyDeviceToHost);
  if (e) return cuda_rc(e);
  err->status = s[0];
  err->first_stream = (int32_t)s[1];
  err->first_step = (int32_t)s[2];
  return LXB_OK;
}

extern "C" int lxb_status_clear(lxb_plan* p) {
  if (!p) return LXB_E_INVAL;
  return cuda_rc(cudaMemset(p->status, 0, 16));
}

extern "C" int lxb_plan_set_profile(lxb_plan* p, unsigned long long* prof) {
  if (!p) return LXB_E_INVAL;
  p->prof = prof;
  return LXB_OK;
}

extern "C" int lxb_profile_sections(void) { return PR_N; }

// An empty cluster barrier's latency: one cluster of `cluster` CTAs (the decode's block size)
// doing nothing but barrier.cluster, timed by rank 0's clock.
__global__ void __launch_bounds__(NT, 1) lxb_cluster_sync_kernel(int iters,
                                                                 unsigned long long* cycles) {
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const long long t0 = clock64();
  for (int i = 0; i < iters; i++) cluster.sync();
  const long long t1 = clock64();
  if (cluster.block_rank() == 0 && threadIdx.x == 0) *cycles = (unsigned long long)(t1 - t0);
}

extern "C" int lxb_cluster_sync_cycles(int cluster, int iters, double* cycles_per_barrier) {
  if (cluster < 1 || cluster > 16 || iters < 1 || !cycles_per_barrier) return LXB_E_INVAL;
  unsigned long long* d = nullptr;
  cudaError_t e = cudaMalloc(&d, sizeof(unsigned long long));
  if (e) return cuda_rc(e);
  if (cluster > 8)
    cudaFuncSetAttribute(lxb_cluster_sync_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(cluster);
  cfg.blockDim = dim3(NT);
  cfg.attrs = at;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, lxb_cluster_sync_kernel, iters, d);
  unsigned long long c = 0;
  if (!e) e = cudaMemcpy(&c, d, sizeof(c), cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e) return cuda_rc(e);
  *cycles_per_barrier = (double)c / iters;
  return LXB_OK;
}

extern "C" int lxb_plan_set_typing(lxb_plan* p, const lxb_typing* ty) {
  if (!p) return LXB_E_INVAL;
  if (!ty || !ty->keys) {
    memset(&p->typing, 0, sizeof(p->typing));
    return LXB_OK;
  }
  if (!ty->n_keys || !ty->tclass || !ty->tstate || ty->max_keys < 0 || ty->rx_slots < 1 ||
      ty->n_class < 0)
    return LXB_E_INVAL;
  p->typing = *ty;
  return LXB_OK;
}

extern "C" int lxb_plan_set_head_helpers(lxb_plan* p, int max_clusters) {
  if (!p || max_clusters < -(LXB_HEADSLICES - LXB_HEADMAIN)) return LXB_E_INVAL;
  p->head_helpers = max_clusters < 0 ? -max_clusters : max_clusters;
  p->help_drill = max_clusters < 0;
  return LXB_OK;
}

extern "C" int lxb_plan_staging(const lxb_plan* p, int* nbuf, int* stage_bytes, int* smem_bytes) {
  if (!p || !nbuf || !stage_bytes || !smem_bytes) return LXB_E_INVAL;
  *nbuf = p->dev.nbuf;
  *stage_bytes = p->dev.stage;
  *smem_bytes = p->smem;
  return LXB_OK;
}

extern "C" size_t lxb_plan_bytes(const lxb_plan* p) { return p ? p->bytes : 0; }
extern "C" int lxb_plan_max_clusters(const lxb_plan* p) { return p ? p->max_clusters : 0; }

extern "C" void lxb_plan_destroy(lxb_plan* p) {
  if (!p) return;
  if (p->dimage) cudaFree(p->dimage);
  if (p->status) cudaFree(p->status);
  delete p;
}
