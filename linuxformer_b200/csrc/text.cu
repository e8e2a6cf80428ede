// Config 5's batch-1 text decode: the Qwen3.5-4B-shaped model (GDN layers zero-padded to the
// chip shape, gated full attention every fourth layer, tied 248,320-row head) as ONE persistent
// cooperative kernel per launch, one CTA per SM, every token's layers and head on the device.
//
// What the kernel computes is the stock forward's decode step (transformers' Qwen3_5 modules,
// modeling_qwen3_5.py: Qwen3_5RMSNorm 711-728, the GDN layer 356-533 with
// torch_causal_conv1d_update 210-226, l2norm 228-231 and torch_recurrent_gated_delta_rule
// 314-353, Qwen3_5Attention 620-693, Qwen3_5MLP 695-709, the decoder layer 731-783), with the
// rounding points of its bf16 tensors; the padding (lx/lx/merge.py:82-120) is skipped by
// construction: the host packs only Qwen's own rows and columns (linuxformer_b200/text.py).
//
// Batch 1 is a chain of matrix-vector products over ~8.4 GB of weights per token, so the design
// is a weight stream: every CTA owns a fixed row range of every matrix, and its producer warp
// issues cp.async.bulk copies of those rows, chunk after chunk, into a ring of NS shared-memory
// stages (full / empty mbarriers per stage). Weights do not depend on the activations, so the
// stream runs ahead of the compute across phases and grid barriers: while the 15 consumer warps
// wait at a barrier or work on a recurrence, the next chunks are already on the way, and a
// producer blocked on the copy engine never holds the consumers up. A row's dot product is
// split into fixed segments, one warp each, added in segment order, so every result is
// independent of how rows are spread over CTAs.
//
// Phases per layer (no grid barrier between them: every activation a phase reads from other CTAs
// is stored with a 16-bit version tag in the same 32-bit word, and the reader polls the words it
// needs until they carry the version it expects; the data dependencies between phases then order
// every overwrite after every read of the version before, and the one grid barrier left is the
// head's):
//   P1  RMSNorm(x) -> the layer's input projections (GDN: q k v z b a; attention: q+gate k v)
//   P2  GDN: conv, l2 norms, gates, the delta rule on the state's live rows (128 CTAs: 32 value
//       heads x 4 column slices) / attention: q/k norm, rope, split-position partial softmax
//       (4 kv heads x G/4 splits), then a combine phase (16 CTAs, one per query head)
//   P3  gated norm (GDN) -> out_proj / o_proj, residual add; the GDN conv windows shift
//   P4  RMSNorm(x) -> gate and up, silu(gate) * up
//   P5  down_proj, residual add
// then the final norm and the head: each CTA's rows' first maximum, the grid's after a barrier.
#include <cuda_runtime.h>
#include <stdint.h>

#include "lxb.h"
#include "lxb_math.h"

namespace {

constexpr int H = 2560, INTER = 9216, VD = 128, QKD = 128, KDP = 256, PR = 8;
constexpr int NKV = 4, HD = 256, ROT = 64;
constexpr int W1G = 12352, W1A = 10240;           // input projection rows (GDN / attention)
constexpr int KOFF = 2048, VOFF = 4096, ZOFF = 8192, BOFF = 12288, AOFF = 12320;
constexpr int KVOFF = 8192, VVOFF = 9216;         // attention: k and v rows of w1
constexpr int NT = 512;                           // 15 consumer warps + the producer warp
constexpr int NCW = 15, NCT = NCW * 32;           // consumers
constexpr int EW = NCW - 1;                       // the consumers' epilogue warp
constexpr int NTASKW = EW;                        // dot-task warps (0 .. 13)
constexpr int SB = 36864;                         // bytes of a ring stage
#ifndef LXB_TEXT_STAGES
#define LXB_TEXT_STAGES 5
#endif
constexpr int NS = LXB_TEXT_STAGES;               // ring stages (consumed in order)
#ifndef LXB_TEXT_LOOKAHEAD
#define LXB_TEXT_LOOKAHEAD 0
#endif
constexpr int LOOKAHEAD = LXB_TEXT_LOOKAHEAD;     // chunks prefetched into L2 beyond the ring
constexpr int APART = 4 + HD;                     // an attention partial: m, l, -, -, acc[256]
constexpr int AACC = 4;                           // (acc 16-byte aligned)
constexpr int NSUB = NCW / 4;                     // attention: position subsets per query head
constexpr long long WAIT_CYCLES = 4000000000ll;   // ~2 s at the B200's clock

struct TP {
  const lxb_text_layer* layers;
  int n_layers, n_vocab, n_embed, max_pos, n_forced, n_tokens, pos0, nsplit;
  float eps;
  const uint16_t* embed;
  const uint16_t* head;
  const uint16_t* fnorm;
  const uint16_t* rope;  // [max_pos][2][64] bf16: cos, sin
  const int32_t* forced;
  int32_t* preds;
  float* hidden;  // optional [n_tokens][n_layers + 1][2560]: each layer's residual, the final norm
  uint32_t *xg, *proj, *vec, *act;  // tagged bf16 activations: residual, projections, mixer out,
                                     // MLP activation (value bits | version tag << 16)
  float *apart, *amax;
  int* aidx;
  unsigned int* acnt;  // attention: arrivals per kv group (the last one combines)
  unsigned long long* bar;
  int* abort_flag;
  uint32_t* status;
  unsigned long long* prof;  // optional [grid][LXB_TEXT_SECTIONS] cycle counters
};

// per-section cycle counters of one CTA (thread 0 keeps them; a null slot turns them off)
struct Prof {
  unsigned long long* slot;
  long long last;
  __device__ __forceinline__ void mark(int k) {
    if (slot && threadIdx.x == 0) {
      const long long now = clock64();
      slot[k] += (unsigned long long)(now - last);
      last = now;
    }
  }
};

struct __align__(128) TSm {
  unsigned char ring[NS][SB];
  uint16_t xb[INTER];  // the phase's input vector (bf16); attention P2 keeps warp partials here
  unsigned long long full[NS], empty[NS];
  float part[2][16];
  float red[16][32];
  float qk[2 * QKD];
  float vv[32], dl[32];
  float aq[4][HD];
  float kn[HD], vn[HD];
  float xres[64];  // this CTA's rows of the residual (it owns them in out_proj and down_proj)
  float bv[16];
  int bi[16];
  float scal[4];
  int tok, abort_seen, tok_last;
};
static_assert(sizeof(TSm) <= 232448, "shared memory");
static_assert(sizeof(float) * 4 * NSUB * APART <= sizeof(uint16_t) * INTER, "attention partials");

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
// the consumers' block barrier (the producer warp runs on its own)
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }
// the same barrier, returning whether v held on every consumer thread
__device__ __forceinline__ bool csync_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, 1, %2, p;\n"
      " selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(NCT)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ float bfv(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }
__device__ __forceinline__ uint16_t bfbits(float bf_valued) {
  return (uint16_t)(__float_as_uint(bf_valued) >> 16);
}
// Tagged activations: a bf16 value and its version's tag in one 32-bit word (single-copy atomic),
// stored and loaded as relaxed gpu-scope operations. Tags are 1..65535 (the buffers are cleared
// to 0 before every launch); a word is rewritten every token, so a stale word's tag is at most a
// token's versions old and never equals the one a reader waits for.
__device__ __forceinline__ uint32_t vtag(long long v) { return 1u + (uint32_t)(v % 65535); }
__device__ __forceinline__ float wval(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ void st_tag(uint32_t* a, float bf_valued, uint32_t tag) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a),
               "r"((__float_as_uint(bf_valued) >> 16) | (tag << 16))
               : "memory");
}
__device__ __forceinline__ uint32_t ld_rel(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_rel4(const uint32_t* a) {
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(a)
               : "memory");
  return v;
}
__device__ __forceinline__ void poll_fail(const TP& p) {
  atomicOr(p.status, LXB_S_SYNC);
  atomicExch(p.abort_flag, 1);
}
// spin until the word carries tag (bounded: ~2 s, or earlier once another CTA aborted)
__device__ __forceinline__ bool poll1(const TP& p, const uint32_t* a, uint32_t tag, float& x) {
  long long t0 = 0;
  for (int it = 0;; it++) {
    const uint32_t v = ld_rel(a);
    if ((v >> 16) == tag) {
      x = wval(v);
      return true;
    }
    if (it == 0) t0 = clock64();
    else if ((it & 255) == 0 && *(volatile const int*)p.abort_flag) return false;
    if (clock64() - t0 > WAIT_CYCLES) {
      poll_fail(p);
      return false;
    }
  }
}
// the same for 4 consecutive words (16-byte aligned)
__device__ __forceinline__ bool poll4(const TP& p, const uint32_t* a, uint32_t tag, float (&x)[4]) {
  long long t0 = 0;
  for (int it = 0;; it++) {
    const uint4 v = ld_rel4(a);
    if ((v.x >> 16) == tag && (v.y >> 16) == tag && (v.z >> 16) == tag && (v.w >> 16) == tag) {
      x[0] = wval(v.x), x[1] = wval(v.y), x[2] = wval(v.z), x[3] = wval(v.w);
      return true;
    }
    if (it == 0) t0 = clock64();
    else if ((it & 255) == 0 && *(volatile const int*)p.abort_flag) return false;
    if (clock64() - t0 > WAIT_CYCLES) {
      poll_fail(p);
      return false;
    }
  }
}
__device__ __forceinline__ void bf8(uint4 v, float (&x)[8]) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; i++) x[2 * i] = __uint_as_float(u[i] << 16), x[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
}
__device__ __forceinline__ float dot8(uint4 w, uint4 x, float a) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w}, xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    a = __fmaf_rn(__uint_as_float(ws[i] << 16), __uint_as_float(xs[i] << 16), a);
    a = __fmaf_rn(__uint_as_float(ws[i] & 0xffff0000u), __uint_as_float(xs[i] & 0xffff0000u), a);
  }
  return a;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// --- the weight stream ----------------------------------------------------------------------
// Phase ph of a token: 4 per layer (w1, wo, wgu, wd), then the head (ph == 4 * n_layers).
struct PhaseDesc {
  const uint16_t* W;
  int n, K, q;
};
__device__ __forceinline__ PhaseDesc pdesc(const TP& p, int ph) {
  if (ph == 4 * p.n_layers) return {p.head, p.n_vocab, H, 1};
  const lxb_text_layer& L = p.layers[ph >> 2];
  switch (ph & 3) {
    case 0: return {(const uint16_t*)L.w1, L.type ? W1A : W1G, H, 1};
    case 1: return {(const uint16_t*)L.wo, H, 4096, 1};
    case 2: return {(const uint16_t*)L.wgu, 2 * INTER, H, 2};  // gate/up row pairs
    default: return {(const uint16_t*)L.wd, H, INTER, 1};
  }
}
// rows of one chunk; a chunk's rows x segments is at most NTASKW dot tasks
__device__ __forceinline__ int rows_per_chunk(int K, int q) {
  return K == H ? (q == 2 ? 6 : 7) : (K == 4096 ? 3 : 2);
}
// a row's dot product is split into segs_of(K) segments of 32 * V 16-byte vectors (V = 5, 4, 6
// for K = 2560, 4096, 9216), one warp each; the segments' sums are added in order
__device__ __forceinline__ int segs_of(int K) { return K == H ? 2 : (K == 4096 ? 4 : 6); }

template <int V>
__device__ __forceinline__ float dot_task(const uint4* wp, const uint4 (&xv)[6], int lane) {
  uint4 wv[V];
#pragma unroll
  for (int i = 0; i < V; i++) wv[i] = wp[i * 32 + lane];
  float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
  for (int i = 0; i < V; i++) {
    if (i & 1) a1 = dot8(wv[i], xv[i], a1);
    else a0 = dot8(wv[i], xv[i], a0);
  }
  return warp_sum(a0 + a1);
}
// CTA c's rows of an n-row matrix (whole groups of q rows), contiguous
__device__ __forceinline__ void rows_of(int n, int q, int c, int G, int& r0, int& r1) {
  const long long u = n / q;
  r0 = (int)(c * u / G) * q;
  r1 = (int)((c + 1) * u / G) * q;
}

__device__ __forceinline__ bool mbar_test(uint32_t mb, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(mb), "r"(parity)
      : "memory");
  return ok;
}
// bounded wait for an mbarrier phase; gives up after ~2 s, or early once the abort flag is set
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity,
                                          const int* abort_flag) {
  const uint32_t mb = smem_u32(bar);
  long long t0 = 0;
  for (int it = 0;; it++) {
    if (mbar_test(mb, parity)) return true;
    if (it == 0) t0 = clock64();
    if ((it & 1023) == 1023 && abort_flag && *(volatile const int*)abort_flag) return false;
    if (clock64() - t0 > WAIT_CYCLES) return false;
  }
}

// the producer's cursor: the next chunk of this CTA's weight stream
struct Prod {
  int tok, ph, a, r1, K, rp;
  const uint16_t* W;
  __device__ void seek(const TP& p) {  // from (tok, ph) to the first phase with rows for this CTA
    const int nph = 4 * p.n_layers + 1;
    while (tok < p.n_tokens) {
      const PhaseDesc d = pdesc(p, ph);
      int r0;
      rows_of(d.n, d.q, blockIdx.x, gridDim.x, r0, r1);
      if (r1 > r0) {
        a = r0;
        K = d.K;
        rp = rows_per_chunk(d.K, d.q);
        W = d.W;
        return;
      }
      if (++ph == nph) ph = 0, tok++;
    }
  }
  __device__ void advance(const TP& p, int nr) {
    a += nr;
    if (a >= r1) {
      if (++ph == 4 * p.n_layers + 1) ph = 0, tok++;
      seek(p);
    }
  }
  // the chunk at the cursor into L2 only, then the cursor moves on
  __device__ void prefetch(const TP& p) {
    if (tok >= p.n_tokens) return;
    const int nr = min(rp, r1 - a);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(W + (size_t)a * K),
                 "r"((uint32_t)nr * K * 2)
                 : "memory");
    advance(p, nr);
  }
  __device__ void issue(const TP& p, TSm& s, int stage) {
    const int nr = min(rp, r1 - a);
    const uint32_t bytes = (uint32_t)nr * K * 2;
    const unsigned char* src = reinterpret_cast<const unsigned char*>(W + (size_t)a * K);
    const uint32_t mb = smem_u32(&s.full[stage]);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mb), "r"(bytes)
                 : "memory");
    for (uint32_t o = 0; o < bytes; o += 32768) {
      const uint32_t nb = min(32768u, bytes - o);
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
          ::"r"(smem_u32(&s.ring[stage][o])), "l"(src + o), "r"(nb), "r"(mb)
          : "memory");
    }
    advance(p, nr);
  }
};

// The producer warp's lane 0: every chunk of every token in order into stage k % NS, once the
// consumers have released that stage (empty barrier). Before it leaves, every copy it issued
// has landed, so no copy writes shared memory after the block is gone.
__device__ void producer(const TP& p, TSm& s) {
  Prod pr{0, 0, 0, 0, 0, 0, nullptr};
  pr.seek(p);
  Prod ahead = pr;  // LOOKAHEAD chunks past the last one issued, into L2
  for (int i = 0; i < LOOKAHEAD; i++) ahead.prefetch(p);
  uint32_t k = 0;
  while (pr.tok < p.n_tokens) {
    const int st = k % NS;
    if (k >= NS && !mbar_wait(&s.empty[st], ((k / NS) + 1) & 1, p.abort_flag)) break;
    pr.issue(p, s, st);
    if (LOOKAHEAD) ahead.prefetch(p);
    k++;
  }
  for (uint32_t j = k > NS ? k - NS : 0; j < k; j++) mbar_wait(&s.full[j % NS], (j / NS) & 1, nullptr);
}

__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* a) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(a) : "memory");
  return v;
}

// grid barrier over a launch-local counter (zeroed before the launch): barrier k completes at
// k * G arrivals. Bounded: a wait past ~2 s sets LXB_S_SYNC and the abort flag, and every CTA
// leaves at its next barrier.
__device__ bool grid_sync(const TP& p, TSm& s, unsigned long long& target) {
  csync();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(p.bar) : "memory");
    long long t0 = clock64();
    int bad = 0;
    while (ld_acquire(p.bar) < target) {
      if (*(volatile int*)p.abort_flag) { bad = 1; break; }
      if (clock64() - t0 > WAIT_CYCLES) {
        atomicOr(p.status, LXB_S_SYNC);
        atomicExch(p.abort_flag, 1);
        bad = 1;
        break;
      }
    }
    if (!bad && *(volatile int*)p.abort_flag) bad = 1;
    s.abort_seen = bad;
  }
  csync();
  return !s.abort_seen;
}

__device__ __forceinline__ void fail_stage(const TP& p) {
  if (threadIdx.x == 0) {
    atomicOr(p.status, LXB_S_STAGE);
    atomicExch(p.abort_flag, 1);
  }
}

// consumer-wide sum in a fixed order: warp butterflies, then warp 0 over the warp sums
__device__ float block_sum(TSm& s, float v) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) s.red[w][0] = v;
  csync();
  float r = lane < NCW ? s.red[lane][0] : 0.0f;
  r = warp_sum(r);
  csync();
  return r;
}

// Qwen3_5RMSNorm of a 2560-vector into s.xb: bf16(x * rsqrt(mean(x^2) + eps) * (1 + w)).
// The vector: the embedding row erow (bf16), or the residual (tagged words of version tag).
// Thread t < 320 takes elements 8t .. 8t + 7. dump (or null): where the vector is copied (the
// per-layer residuals of `hidden`). Returns false (on every consumer thread) after a failed poll.
__device__ bool norm_to_xb(const TP& p, TSm& s, const uint16_t* erow, uint32_t tag,
                           const uint16_t* w, float* dump = nullptr) {
  const int t = threadIdx.x;
  float x[8], ss = 0.0f;
  const bool on = t < H / 8;
  bool ok = true;
  if (on) {
    if (erow) {
      bf8(__ldg(reinterpret_cast<const uint4*>(erow) + t), x);
    } else {
      float a[4], b[4];
      ok = poll4(p, p.xg + 8 * t, tag, a) && poll4(p, p.xg + 8 * t + 4, tag, b);
#pragma unroll
      for (int i = 0; i < 4; i++) x[i] = a[i], x[4 + i] = b[i];
    }
#pragma unroll
    for (int i = 0; i < 8; i++) ss = lx_add(ss, lx_mul(x[i], x[i]));
    if (dump)
#pragma unroll
      for (int i = 0; i < 8; i++) dump[8 * t + i] = x[i];
  }
  if (!csync_and(ok)) return false;
  const float tot = block_sum(s, ss);
  const float r = lx_rsqrt(lx_add(lx_div(tot, (float)H), p.eps));
  if (on) {
    float wf[8];
    bf8(*(reinterpret_cast<const uint4*>(w) + t), wf);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; i++)
      o[i] = (uint32_t)lx_rb(lx_mul(lx_mul(x[2 * i], r), lx_add(1.0f, wf[2 * i]))) |
             ((uint32_t)lx_rb(lx_mul(lx_mul(x[2 * i + 1], r), lx_add(1.0f, wf[2 * i + 1]))) << 16);
    reinterpret_cast<uint4*>(s.xb)[t] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  return true;
}

// n tagged words (n a multiple of 4) of version tag into s.xb as bf16; false after a failed poll
__device__ bool copy_to_xb(const TP& p, TSm& s, const uint32_t* src, int n, uint32_t tag) {
  bool ok = true;
  for (int i = threadIdx.x; ok && i < n / 4; i += NCT) {
    float v[4];
    ok = poll4(p, src + 4 * i, tag, v);
    reinterpret_cast<uint2*>(s.xb)[i] =
        make_uint2((__float_as_uint(v[0]) >> 16) | (__float_as_uint(v[1]) & 0xffff0000u),
                   (__float_as_uint(v[2]) >> 16) | (__float_as_uint(v[3]) & 0xffff0000u));
  }
  return csync_and(ok);
}

enum { EP_PROJ = 0, EP_RESID = 1, EP_ACT = 2, EP_HEAD = 3 };

// One phase of the weight stream: this CTA's rows of matrix ph times s.xb. Every chunk has at
// most NTASKW dot tasks (rows x segments), task k on warp k: a warp's row and segment are the
// same in every chunk of the phase, so its part of the input vector stays in registers. The
// epilogue (segment sums, rounding, stores) runs on warp EW. A staging timeout sets the abort
// flag, which the next grid barrier reads.
__device__ void gemv(const TP& p, TSm& s, Prof& pf, uint32_t& cc, int ph, int ep, uint32_t tag,
                     float& bestv, int& besti) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, et = t - EW * 32;
  const PhaseDesc d = pdesc(p, ph);
  int r0, r1;
  rows_of(d.n, d.q, blockIdx.x, gridDim.x, r0, r1);
  const int rp = rows_per_chunk(d.K, d.q), nsg = segs_of(d.K), V = d.K / (256 * nsg);
  csync();  // s.xb complete
  const int wr = w / nsg, wsg = w - wr * nsg;
  uint4 xv[6];
  {
    const uint4* xp = reinterpret_cast<const uint4*>(s.xb) + wsg * 32 * V;
#pragma unroll
    for (int i = 0; i < 6; i++)
      xv[i] = (i < V && w < NTASKW) ? xp[i * 32 + lane] : make_uint4(0, 0, 0, 0);
  }
  for (int a = r0; a < r1; a += rp) {
    const int nr = min(rp, r1 - a), stage = cc % NS;
    pf.mark(LXB_TP_GEMV);
    const bool landed = mbar_wait(&s.full[stage], (cc / NS) & 1, p.abort_flag);
    pf.mark(LXB_TP_WAIT);
    float* part = s.part[cc & 1];
    if (landed && w < nr * nsg) {
      const uint4* wp = reinterpret_cast<const uint4*>(s.ring[stage] + (size_t)wr * d.K * 2) +
                        wsg * 32 * V;
      const float acc = V == 5 ? dot_task<5>(wp, xv, lane)
                               : (V == 4 ? dot_task<4>(wp, xv, lane) : dot_task<6>(wp, xv, lane));
      if (lane == 0) part[w] = acc;
    }
    if (!csync_and(landed)) {  // a copy that never landed: every consumer leaves together
      fail_stage(p);
      break;
    }
    if (t == 0)  // the stage is free for the producer
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&s.empty[stage]))
                   : "memory");
    if (ep == EP_ACT) {
      if (et >= 0 && et < nr / 2) {
        float yg = 0.0f, yu = 0.0f;
        for (int sg = 0; sg < nsg; sg++) {
          yg = lx_add(yg, part[(2 * et) * nsg + sg]);
          yu = lx_add(yu, part[(2 * et + 1) * nsg + sg]);
        }
        const float g = lx_rbf(yg), u = lx_rbf(yu);
        st_tag(p.act + a / 2 + et, lx_rbf(lx_mul(lx_rbf(lx_silu(g)), u)), tag);
      }
    } else if (et >= 0 && et < nr) {
      float y = 0.0f;
      for (int sg = 0; sg < nsg; sg++) y = lx_add(y, part[et * nsg + sg]);
      const int row = a + et;
      if (ep == EP_PROJ) {
        st_tag(p.proj + row, lx_rbf(y), tag);
      } else if (ep == EP_RESID) {
        const float x = lx_rbf(lx_add(s.xres[row - r0], lx_rbf(y)));
        s.xres[row - r0] = x;  // only this thread touches this row in the phase
        st_tag(p.xg + row, x, tag);
      } else {
        const float v = lx_rbf(y);
        if (v > bestv) bestv = v, besti = row;
      }
    }
    cc++;
  }
  pf.mark(LXB_TP_GEMV);
}

// --- P2: the GDN step of one (value head, 32-column slice) --------------------------------------
__device__ bool gdn_p2(const TP& p, TSm& s, const lxb_text_layer& L, int task, uint32_t tag) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int vh = task >> 2, sl = task & 3, kh = vh >> 1, ph = kh * PR + (vh & 1);
  const uint16_t* cw = (const uint16_t*)L.conv_w;
  const uint16_t* cs = (const uint16_t*)L.conv_state;
  // the state's live rows 0..127 of this column slice (warp w < 8: rows 16w .. 16w + 15),
  // loaded first: their address depends on nothing computed here
  float* S = (float*)L.rec_state + (size_t)ph * KDP * VD + sl * 32 + lane;
  float h[16];
  if (w < 8)
#pragma unroll
    for (int i = 0; i < 16; i++) h[i] = __ldcg(S + (size_t)(w * 16 + i) * VD);
  // the conv windows were written by other CTAs at earlier tokens: everything they stored before
  // the tagged words this CTA has since seen from them is visible after this fence
  __threadfence();
  bool ok = true;
  if (t == 288 || t == 289) ok = poll1(p, p.proj + (t == 288 ? BOFF : AOFF) + vh, tag, s.scal[t - 286]);
  // conv over the new window [w1 w2 w3 P] (torch_causal_conv1d_update), silu, bf16
  if (t < 288) {
    int prow, pch;
    if (t < 128) prow = kh * QKD + t, pch = kh * KDP + t;
    else if (t < 256) prow = KOFF + kh * QKD + (t - 128), pch = 16 * KDP + kh * KDP + (t - 128);
    else {
      const int j = sl * 32 + (t - 256);
      prow = VOFF + vh * VD + j;
      pch = 2 * 16 * KDP + ph * VD + j;
    }
    float P = 0.0f;
    ok = poll1(p, p.proj + prow, tag, P);
    const uint2 win = __ldcg(reinterpret_cast<const uint2*>(cs + (size_t)pch * 4));
    const uint2 tap = *reinterpret_cast<const uint2*>(cw + (size_t)prow * 4);
    float y = 0.0f;
    y = lx_add(y, lx_mul(bfv(tap.x & 0xffff), bfv(win.x >> 16)));
    y = lx_add(y, lx_mul(bfv(tap.x >> 16), bfv(win.y & 0xffff)));
    y = lx_add(y, lx_mul(bfv(tap.y & 0xffff), bfv(win.y >> 16)));
    y = lx_add(y, lx_mul(bfv(tap.y >> 16), P));
    const float o = lx_rbf(lx_silu(lx_rbf(y)));
    if (t < 256) s.qk[t] = o;
    else s.vv[t - 256] = o;
  }
  if (!csync_and(ok)) return false;
  // l2norm in bf16 (q by warp 0, k by warp 1; q then times 256^-0.5, exact), beta and decay
  if (w < 2) {
    float x[4], sq = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      x[i] = s.qk[w * QKD + lane * 4 + i];
      sq = lx_add(sq, lx_rbf(lx_mul(x[i], x[i])));
    }
    sq = warp_sum(sq);
    const float se = lx_rbf(lx_add(lx_rbf(sq), 1e-6f));
    const float inv = lx_rbf(lx_rsqrt(se));
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float n = lx_rbf(lx_mul(x[i], inv));
      s.qk[w * QKD + lane * 4 + i] = w == 0 ? lx_mul(n, 0.0625f) : n;
    }
  } else if (t == 64) {
    const float b = s.scal[2], a = s.scal[3];
    const float beta = lx_rbf(lx_sigmoid(b));
    const float A = -lx_exp(((const float*)L.A_log)[vh]);
    const float g = lx_mul(A, lx_softplus(lx_add(a, ((const float*)L.dt_bias)[vh])));
    s.scal[0] = beta;
    s.scal[1] = lx_exp(g);
  }
  csync();
  const float beta = s.scal[0], e = s.scal[1];
  if (w < 8) {
    float kv = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      h[i] = lx_mul(h[i], e);
      kv = lx_add(kv, lx_mul(h[i], s.qk[QKD + w * 16 + i]));
    }
    s.red[w][lane] = kv;
  }
  csync();
  if (w == 0) {
    float k2 = 0.0f;
    for (int g2 = 0; g2 < 8; g2++) k2 = lx_add(k2, s.red[g2][lane]);
    s.dl[lane] = lx_mul(lx_sub(s.vv[lane], k2), beta);
  }
  csync();
  if (w < 8) {
    const float delta = s.dl[lane];
    float o = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const int r = w * 16 + i;
      h[i] = lx_add(h[i], lx_mul(s.qk[QKD + r], delta));
      o = lx_add(o, lx_mul(h[i], s.qk[r]));
      __stcg(S + (size_t)r * VD, h[i]);
    }
    s.red[w][lane] = o;
  }
  csync();
  if (w == 0) {
    float o2 = 0.0f;
    for (int g2 = 0; g2 < 8; g2++) o2 = lx_add(o2, s.red[g2][lane]);
    st_tag(p.vec + vh * VD + sl * 32 + lane, lx_rbf(o2), tag);
  }
  csync();
  return true;
}

// P3 of a GDN layer: the conv windows of this CTA's channels shift in the new projection
__device__ bool gdn_windows(const TP& p, const lxb_text_layer& L, uint32_t tag) {
  bool ok = true;
  const int G = gridDim.x, c = blockIdx.x;
  const int c0 = (int)((long long)c * 8192 / G), c1 = (int)((long long)(c + 1) * 8192 / G);
  uint16_t* cs = (uint16_t*)L.conv_state;
  for (int ch = c0 + (int)threadIdx.x; ch < c1; ch += NCT) {
    int pch;
    if (ch < KOFF) pch = (ch >> 7) * KDP + (ch & 127);
    else if (ch < VOFF) pch = 16 * KDP + ((ch - KOFF) >> 7) * KDP + (ch & 127);
    else {
      const int vh = (ch - VOFF) >> 7;
      pch = 2 * 16 * KDP + ((vh >> 1) * PR + (vh & 1)) * VD + (ch & 127);
    }
    uint2* wp = reinterpret_cast<uint2*>(cs + (size_t)pch * 4);
    const uint2 win = __ldcg(wp);
    float Pv;
    if (!(ok = poll1(p, p.proj + ch, tag, Pv))) break;
    const uint32_t P = __float_as_uint(Pv) >> 16;
    __stcg(wp, make_uint2((win.x >> 16) | (win.y << 16), (win.y >> 16) | (P << 16)));
  }
  __threadfence();  // the windows before any tagged word this CTA stores later
  return ok;
}

// P3 of a GDN layer: Qwen3_5RMSNormGated of the 32 heads' outputs into s.xb:
// bf16(bf16(w * bf16(o * rsqrt(mean(o^2) + eps))) * silu(z)), the product with w unrounded when w
// is an fp32 parameter
__device__ bool gdn_gated_norm(const TP& p, TSm& s, const lxb_text_layer& L, uint32_t tag,
                               bool ok) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const float* gw = (const float*)L.gnorm;
  const bool gf32 = L.flags & LXB_TEXT_GNORM_F32;
  for (int vh = w; vh < 32; vh += NCW) {
    float o[4], z4[4], sq = 0.0f;
    ok = ok && poll4(p, p.vec + vh * VD + lane * 4, tag, o) &&
         poll4(p, p.proj + ZOFF + vh * VD + lane * 4, tag, z4);
    if (__any_sync(0xffffffffu, !ok)) break;
#pragma unroll
    for (int i = 0; i < 4; i++) sq = lx_add(sq, lx_mul(o[i], o[i]));
    sq = warp_sum(sq);
    const float rr = lx_rsqrt(lx_add(lx_div(sq, 128.0f), p.eps));
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int j = lane * 4 + i;
      const float hn = lx_rbf(lx_mul(o[i], rr));
      const float u = gf32 ? lx_mul(gw[j], hn) : lx_rbf(lx_mul(gw[j], hn));
      s.xb[vh * VD + j] = lx_rb(lx_mul(u, lx_silu(z4[i])));
    }
  }
  return csync_and(ok);
}

// --- P2 of an attention layer: one (kv head, position split) ------------------------------------
// nh heads (nh <= 4), head k from src + k * stride into dst + k * HD, 64 threads a head (4 dims
// each): RMSNorm over the head's 256 dims (q_norm / k_norm), then rope on the first 64 dims with
// bf16 rounding after every tensor op (apply_rotary_pos_emb, modeling_qwen3_5.py:544-579)
__device__ bool head_norm_rope(const TP& p, TSm& s, float* dst, const uint32_t* src, int stride,
                               const uint16_t* w, int pos, int nh, uint32_t tag) {
  const int t = threadIdx.x, grp = t >> 6, d0 = (t & 63) * 4;
  const bool on = t < nh * 64;
  float x[4] = {0.0f, 0.0f, 0.0f, 0.0f}, ss = 0.0f;
  bool ok = true;
  if (on) {
    ok = poll4(p, src + grp * stride + d0, tag, x);
#pragma unroll
    for (int i = 0; i < 4; i++) ss = lx_add(ss, lx_mul(x[i], x[i]));
  }
  ss = warp_sum(ss);
  if ((t & 31) == 0 && t < 256) s.red[t >> 5][1] = ss;
  if (!csync_and(ok)) return false;
  float* o = dst + grp * HD;
  if (on) {
    const float tot = lx_add(s.red[2 * grp][1], s.red[2 * grp + 1][1]);
    const float r = lx_rsqrt(lx_add(lx_div(tot, (float)HD), p.eps));
#pragma unroll
    for (int i = 0; i < 4; i++)
      o[d0 + i] = lx_rbf(lx_mul(lx_mul(x[i], r), lx_add(1.0f, bfv(w[d0 + i]))));
  }
  csync();
  float nv[4];
  const bool rot = on && d0 < ROT;
  if (rot) {
    const uint16_t* cs = p.rope + (size_t)pos * 2 * ROT;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int d = d0 + i;
      const float xv = o[d], rh = d < ROT / 2 ? -o[d + ROT / 2] : o[d - ROT / 2];
      nv[i] = lx_rbf(lx_add(lx_rbf(lx_mul(xv, bfv(cs[d]))), lx_rbf(lx_mul(rh, bfv(cs[ROT + d])))));
    }
  }
  csync();
  if (rot)
#pragma unroll
    for (int i = 0; i < 4; i++) o[d0 + i] = nv[i];
  csync();
  return true;
}

// The combine: kv group g's 4 query heads over all splits in order, softmax-normalised, times
// sigmoid(gate) (every split's m and l staged in shared memory first, then each output's
// accumulators with their loads in flight together)
__device__ bool att_combine(const TP& p, TSm& s, int g, uint32_t tag) {
  bool ok = true;
  const int t = threadIdx.x, ns = p.nsplit;
  float* ms = &s.aq[0][0];  // [4][ns]
  float* ls = ms + 4 * ns;
  float* fs = ls + 4 * ns;
  const float* base = p.apart + (size_t)(g * ns) * 4 * APART;  // split sp, head h4: (sp*4+h4)
  for (int k = t; k < 4 * ns; k += NCT) {
    const int h4 = k / ns, sp = k % ns;
    ms[k] = __ldcg(base + (size_t)(sp * 4 + h4) * APART);
    ls[k] = __ldcg(base + (size_t)(sp * 4 + h4) * APART + 1);
  }
  csync();
  for (int k = t; k < 4 * ns; k += NCT) {
    const int h4 = k / ns;
    float M = -INFINITY;
    for (int sp = 0; sp < ns; sp++) M = fmaxf(M, ms[h4 * ns + sp]);
    fs[k] = ms[k] == -INFINITY ? 0.0f : lx_exp(lx_sub(ms[k], M));
  }
  csync();
  // 4 heads x 64 groups of 4 dims, one a thread: every split's 4 accumulators as one 16-byte
  // load, 8 splits' loads in flight together
  for (int k = t; k < HD; k += NCT) {
    const int h4 = k / (HD / 4), d = (k % (HD / 4)) * 4;
    float Ls = 0.0f, A[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int s0 = 0; s0 < ns; s0 += 8) {
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; j++)
        v[j] = s0 + j < ns ? __ldcg(reinterpret_cast<const float4*>(
                                 base + (size_t)((s0 + j) * 4 + h4) * APART + AACC + d))
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int j = 0; j < 8; j++)
        if (s0 + j < ns) {
          const float f = fs[h4 * ns + s0 + j];
          Ls = __fmaf_rn(ls[h4 * ns + s0 + j], f, Ls);
          A[0] = __fmaf_rn(v[j].x, f, A[0]);
          A[1] = __fmaf_rn(v[j].y, f, A[1]);
          A[2] = __fmaf_rn(v[j].z, f, A[2]);
          A[3] = __fmaf_rn(v[j].w, f, A[3]);
        }
    }
    const int h = g * 4 + h4;
    float gate[4];
    ok = ok && poll4(p, p.proj + h * 2 * HD + HD + d, tag, gate);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float o = lx_rbf(lx_div(A[i], Ls));
      st_tag(p.vec + h * HD + d + i, lx_rbf(lx_mul(o, lx_rbf(lx_sigmoid(gate[i])))), tag);
    }
  }
  return csync_and(ok);
}

__device__ bool att_p2(const TP& p, TSm& s, const lxb_text_layer& L, int pos, uint32_t tag) {
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int ns = p.nsplit, g = blockIdx.x / ns, sp = blockIdx.x % ns;
  const long long n = pos + 1;
  const int b0 = (int)(sp * n / ns), b1 = (int)((sp + 1) * n / ns);
  const bool last = sp == ns - 1;
  // the key/value rows were written by other CTAs at earlier tokens: visible after this fence
  __threadfence();
  // the group's 4 query heads, then the new key and value (if this split holds pos)
  if (!head_norm_rope(p, s, &s.aq[0][0], p.proj + (g * 4) * 2 * HD, 2 * HD,
                      (const uint16_t*)L.qn, pos, 4, tag))
    return false;
  if (last) {
    if (!head_norm_rope(p, s, s.kn, p.proj + KVOFF + g * HD, 0, (const uint16_t*)L.kn, pos, 1,
                        tag))
      return false;
    bool ok = true;
    if (t < HD) ok = poll1(p, p.proj + VVOFF + g * HD + t, tag, s.vn[t]);
    if (!csync_and(ok)) return false;
  }
  // warp w < 4 * NSUB: query head hh = w & 3 over the positions b0 + ss + NSUB * j
  // (ss = w >> 2), four of them per round with their loads in flight together; lane: dims
  // 8 * lane .. + 8
  float* aw = reinterpret_cast<float*>(s.xb);  // [4 * NSUB warps][APART]
  if (w < 4 * NSUB) {
    const int hh = w & 3, ss = w >> 2;
    float qv[8], acc[8], m = -INFINITY, l = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) qv[i] = s.aq[hh][lane * 8 + i], acc[i] = 0.0f;
    const uint16_t* kc = (const uint16_t*)L.kc + (size_t)g * p.max_pos * HD;
    const uint16_t* vc = (const uint16_t*)L.vc + (size_t)g * p.max_pos * HD;
    for (int q0 = b0 + ss; q0 < b1; q0 += 4 * NSUB) {
      uint4 kw[4], vw[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int q = q0 + NSUB * j;
        if (q < b1 && q != pos) {
          kw[j] = __ldcg(reinterpret_cast<const uint4*>(kc + (size_t)q * HD) + lane);
          vw[j] = __ldcg(reinterpret_cast<const uint4*>(vc + (size_t)q * HD) + lane);
        } else {
          kw[j] = make_uint4(0, 0, 0, 0);
          vw[j] = kw[j];
        }
      }
      float sc[4], vx[4][8];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int q = q0 + NSUB * j;
        float kx[8];
        if (q == pos) {
#pragma unroll
          for (int i = 0; i < 8; i++) kx[i] = s.kn[lane * 8 + i], vx[j][i] = s.vn[lane * 8 + i];
        } else {
          const uint32_t ka[4] = {kw[j].x, kw[j].y, kw[j].z, kw[j].w};
          const uint32_t va[4] = {vw[j].x, vw[j].y, vw[j].z, vw[j].w};
#pragma unroll
          for (int i = 0; i < 4; i++) {
            kx[2 * i] = __uint_as_float(ka[i] << 16);
            kx[2 * i + 1] = __uint_as_float(ka[i] & 0xffff0000u);
            vx[j][2 * i] = __uint_as_float(va[i] << 16);
            vx[j][2 * i + 1] = __uint_as_float(va[i] & 0xffff0000u);
          }
        }
        float dq = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; i++) dq = __fmaf_rn(qv[i], kx[i], dq);
        sc[j] = dq;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < 4; j++) sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], o);
      float mn = m;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        sc[j] = q0 + NSUB * j < b1 ? lx_mul(sc[j], 0.0625f) : -INFINITY;  // head_dim^-0.5
        mn = fmaxf(mn, sc[j]);
      }
      const float alpha = m == -INFINITY ? 0.0f : lx_exp(lx_sub(m, mn));
      l = lx_mul(l, alpha);
#pragma unroll
      for (int i = 0; i < 8; i++) acc[i] = lx_mul(acc[i], alpha);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        if (sc[j] == -INFINITY) continue;
        const float pe = lx_exp(lx_sub(sc[j], mn));
        l = lx_add(l, pe);
#pragma unroll
        for (int i = 0; i < 8; i++) acc[i] = __fmaf_rn(pe, vx[j][i], acc[i]);
      }
      m = mn;
    }
    if (lane == 0) aw[w * APART] = m, aw[w * APART + 1] = l;
#pragma unroll
    for (int i = 0; i < 8; i++) aw[w * APART + AACC + lane * 8 + i] = acc[i];
  }
  csync();
  // the NSUB position subsets of each query head, in order, into this split's partial
  for (int k = t; k < 4 * HD; k += NCT) {
    const int h4 = k / HD, d = k % HD;
    float M = -INFINITY;
    for (int q = 0; q < NSUB; q++) M = fmaxf(M, aw[(q * 4 + h4) * APART]);
    float Ls = 0.0f, A = 0.0f;
    if (M != -INFINITY)
      for (int q = 0; q < NSUB; q++) {
        const float mq = aw[(q * 4 + h4) * APART];
        if (mq == -INFINITY) continue;
        const float f = lx_exp(lx_sub(mq, M));
        Ls = __fmaf_rn(aw[(q * 4 + h4) * APART + 1], f, Ls);
        A = __fmaf_rn(aw[(q * 4 + h4) * APART + AACC + d], f, A);
      }
    float* dst = p.apart + ((size_t)(g * ns + sp) * 4 + h4) * APART;
    if (d == 0) __stcg(dst, M), __stcg(dst + 1, Ls);
    __stcg(dst + AACC + d, A);
  }
  if (last && t < HD) {  // the new key and value join the cache for later tokens
    ((uint16_t*)L.kc)[((size_t)g * p.max_pos + pos) * HD + t] = bfbits(s.kn[t]);
    ((uint16_t*)L.vc)[((size_t)g * p.max_pos + pos) * HD + t] = bfbits(s.vn[t]);
  }
  // the split that arrives last for this kv group combines its 4 query heads (the partials of
  // the others are visible: each CTA fenced its stores before its arrival)
  __threadfence();
  csync();
  if (t == 0) s.tok_last = (int)(atomicAdd(p.acnt + g, 1u) % (unsigned)ns) == ns - 1;
  csync();
  if (s.tok_last) {
    __threadfence();
    return att_combine(p, s, g, tag);
  }
  return true;
}

// first maximum: larger value, or equal value at a lower index
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__global__ void __launch_bounds__(NT, 1) lxb_text_kernel(const TP p) {
  extern __shared__ __align__(128) unsigned char smraw[];
  TSm& s = *reinterpret_cast<TSm*>(smraw);
  const int t = threadIdx.x, lane = t & 31, w = t >> 5, G = gridDim.x, c = blockIdx.x;
  if (t == 0) {
    for (int i = 0; i < NS; i++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&s.full[i])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&s.empty[i])));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s.abort_seen = 0;
  }
  __syncthreads();
  if (w == NCW) {  // the producer warp
    if (lane == 0) producer(p, s);
    return;
  }
  uint32_t cc = 0;
  unsigned long long target = 0;
  Prof pf{p.prof ? p.prof + (size_t)c * LXB_TEXT_SECTIONS : nullptr, clock64()};
  int wo0, wo1;
  rows_of(H, 1, c, G, wo0, wo1);
  for (int it = 0; it < p.n_tokens; it++) {
    const int pos = p.pos0 + it;
    int tok = it < p.n_forced ? p.forced[it] : s.tok;
    if (tok < 0 || tok >= p.n_embed) {
      if (c == 0 && t == 0) atomicOr(p.status, LXB_S_TOKEN);
      tok = min(max(tok, 0), p.n_embed - 1);
    }
    const uint16_t* erow = p.embed + (size_t)tok * H;
    float* hid = p.hidden && c == 0 ? p.hidden + (size_t)it * (p.n_layers + 1) * H : nullptr;
    float bestv = -INFINITY;
    int besti = 0x7fffffff;
    // versions of this token: x at 2 li + 1 after layer li's out_proj, 2 li + 2 after its
    // down_proj; the projections, the mixer output and the MLP activation at the layer's index
    const long long xv0 = (long long)it * (2 * p.n_layers + 1);
    for (int li = 0; li < p.n_layers; li++) {
      const lxb_text_layer& L = p.layers[li];
      const uint32_t tl = vtag((long long)it * p.n_layers + li);
      bool ok;
      if (li == 0) {  // the embedding row: this CTA's residual rows, and the input norm's source
        for (int r = wo0 + t; r < wo1; r += NCT) s.xres[r - wo0] = bfv(erow[r]);
        ok = norm_to_xb(p, s, erow, 0, (const uint16_t*)L.ln_in);
      } else {
        ok = norm_to_xb(p, s, nullptr, vtag(xv0 + 2 * li), (const uint16_t*)L.ln_in,
                        hid ? hid + (size_t)(li - 1) * H : nullptr);
      }
      if (!ok) goto done;
      pf.mark(LXB_TP_NORM);
      gemv(p, s, pf, cc, 4 * li, EP_PROJ, tl, bestv, besti);
      if (L.type == 0) {
        for (int task = c; task < 128; task += G)
          if (!gdn_p2(p, s, L, task, tl)) goto done;
        pf.mark(LXB_TP_GDN);
        // the gated norm first: once this CTA has seen every head's output of the layer, every
        // GDN step has read the old conv windows (its output depends on them), so they may shift
        ok = gdn_gated_norm(p, s, L, tl, true) && csync_and(gdn_windows(p, L, tl));
      } else {
        if (c < NKV * p.nsplit && !att_p2(p, s, L, pos, tl)) goto done;
        pf.mark(LXB_TP_ATT);
        ok = copy_to_xb(p, s, p.vec, 4096, tl);
      }
      if (!ok) goto done;
      pf.mark(LXB_TP_NORM);
      gemv(p, s, pf, cc, 4 * li + 1, EP_RESID, vtag(xv0 + 2 * li + 1), bestv, besti);
      if (!norm_to_xb(p, s, nullptr, vtag(xv0 + 2 * li + 1), (const uint16_t*)L.ln_post)) goto done;
      pf.mark(LXB_TP_NORM);
      gemv(p, s, pf, cc, 4 * li + 2, EP_ACT, tl, bestv, besti);
      if (!copy_to_xb(p, s, p.act, INTER, tl)) goto done;
      pf.mark(LXB_TP_NORM);
      gemv(p, s, pf, cc, 4 * li + 3, EP_RESID, vtag(xv0 + 2 * li + 2), bestv, besti);
    }
    if (!norm_to_xb(p, s, nullptr, vtag(xv0 + 2 * p.n_layers), p.fnorm,
                    hid ? hid + (size_t)(p.n_layers - 1) * H : nullptr))
      goto done;
    if (hid) {
      csync();
      for (int i = t; i < H; i += NCT) hid[(size_t)p.n_layers * H + i] = bfv(s.xb[i]);
    }
    pf.mark(LXB_TP_NORM);
    gemv(p, s, pf, cc, 4 * p.n_layers, EP_HEAD, 0, bestv, besti);
    // this CTA's first maximum, then the grid's (CTAs hold ascending row ranges)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bestv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
      if (better(ov, oi, bestv, besti)) bestv = ov, besti = oi;
    }
    if (lane == 0) s.bv[w] = bestv, s.bi[w] = besti;
    csync();
    if (t == 0) {
      float bv = s.bv[0];
      int bi = s.bi[0];
      for (int k = 1; k < NCW; k++)
        if (better(s.bv[k], s.bi[k], bv, bi)) bv = s.bv[k], bi = s.bi[k];
      __stcg(p.amax + c, bv);
      __stcg(p.aidx + c, bi);
    }
    pf.mark(LXB_TP_HEAD);
    if (!grid_sync(p, s, target)) goto done;
    pf.mark(LXB_TP_SYNC);
    if (w == 0) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int k = lane; k < G; k += 32) {
        const float v = __ldcg(p.amax + k);
        const int i = __ldcg(p.aidx + k);
        if (better(v, i, bv, bi)) bv = v, bi = i;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) bv = ov, bi = oi;
      }
      if (lane == 0) {
        s.tok = bi == 0x7fffffff ? 0 : bi;
        if (c == 0) p.preds[it] = s.tok;
      }
    }
    csync();
    pf.mark(LXB_TP_HEAD);
    if (pf.slot && t == 0) pf.slot[LXB_TP_TOKENS]++;
  }
done:
  // consumers leave here; after an abort the producer warp stops at its next wait and stays
  // until its own copies have landed
  return;
}

}  // namespace

struct lxb_text_plan_s {
  lxb_text_layer* d_layers;
  int n_layers, n_vocab, n_embed, max_pos, device, grid, smem, nsplit;
  float eps;
  const uint16_t *embed, *head, *fnorm, *rope;
  uint32_t* d_status;
  unsigned long long* prof;
};

namespace {
size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }
struct Layout {
  size_t bar, xg, proj, vec, act, apart, amax, aidx, total;
};
Layout layout(const lxb_text_plan* P) {
  Layout l{};
  size_t o = 0;
  l.bar = o;  // bar (u64), abort flag, attention arrival counters [4]
  o = align256(o + 64);
  l.xg = o;  // the tagged words (cleared before every launch): xg, proj, vec, act
  o = align256(o + 4 * H);
  l.proj = o;
  o = align256(o + 4 * W1G);
  l.vec = o;
  o = align256(o + 4 * 4096);
  l.act = o;
  o = align256(o + 4 * INTER);
  l.apart = o;
  o = align256(o + sizeof(float) * NKV * P->nsplit * 4 * APART);
  l.amax = o;
  o = align256(o + sizeof(float) * P->grid);
  l.aidx = o;
  o = align256(o + sizeof(int) * P->grid);
  l.total = o;
  return l;
}
bool al16(uint64_t p) { return p && (p & 15) == 0; }
}  // namespace

extern "C" int lxb_text_plan_create(const lxb_text_layer* layers, int n_layers, const void* embed,
                                    int n_embed, const void* head, int n_vocab,
                                    const void* final_norm, const void* rope, int max_pos,
                                    float eps, int device, lxb_text_plan** out) {
  if (!layers || !out || n_layers < 1 || n_vocab < 1 || n_embed < 1 || max_pos < 1 || !rope ||
      !final_norm || !al16((uint64_t)embed) || !al16((uint64_t)head) || !(eps >= 0.0f))
    return LXB_E_INVAL;
  *out = nullptr;
  for (int i = 0; i < n_layers; i++) {
    const lxb_text_layer& L = layers[i];
    if (L.type != 0 && L.type != 1) return LXB_E_INVAL;
    if (!al16(L.w1) || !al16(L.wo) || !al16(L.wgu) || !al16(L.wd) || !L.ln_in || !L.ln_post)
      return LXB_E_INVAL;
    if (L.type == 0 && (!al16(L.conv_w) || !L.A_log || !L.dt_bias || !L.gnorm ||
                        !al16(L.conv_state) || !al16(L.rec_state)))
      return LXB_E_INVAL;
    if (L.type == 1 && (!L.qn || !L.kn || !al16(L.kc) || !al16(L.vc))) return LXB_E_INVAL;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return LXB_E_DEVICE;
  if (prop.major < 10 || !prop.cooperativeLaunch) return LXB_E_DEVICE;
  int cur = 0;
  cudaGetDevice(&cur);
  cudaSetDevice(device);
  const int smem = (int)sizeof(TSm);
  int per_sm = 0;
  cudaError_t e = cudaFuncSetAttribute(lxb_text_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem);
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, lxb_text_kernel, NT, smem);
  if (e != cudaSuccess || per_sm < 1 || prop.multiProcessorCount < 64) {
    cudaSetDevice(cur);
    return LXB_E_DEVICE;
  }
  auto* P = new lxb_text_plan_s{};
  P->n_layers = n_layers;
  P->n_vocab = n_vocab;
  P->n_embed = n_embed;
  P->max_pos = max_pos;
  P->device = device;
  P->grid = prop.multiProcessorCount;  // one CTA per SM (the ring fills the shared memory)
  P->nsplit = P->grid / NKV;
  P->smem = smem;
  P->eps = eps;
  P->embed = (const uint16_t*)embed;
  P->head = (const uint16_t*)head;
  P->fnorm = (const uint16_t*)final_norm;
  P->rope = (const uint16_t*)rope;
  e = cudaMalloc(&P->d_layers, sizeof(lxb_text_layer) * n_layers);
  if (e == cudaSuccess)
    e = cudaMemcpy(P->d_layers, layers, sizeof(lxb_text_layer) * n_layers, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&P->d_status, 16);
  if (e == cudaSuccess) e = cudaMemset(P->d_status, 0, 16);
  cudaSetDevice(cur);
  if (e != cudaSuccess) {
    lxb_text_plan_destroy(P);
    return (int)e;
  }
  *out = P;
  return 0;
}

extern "C" size_t lxb_text_scratch_bytes(const lxb_text_plan* P) {
  return P ? layout(P).total : 0;
}

extern "C" int lxb_text_decode(lxb_text_plan* P, const int32_t* forced, int n_forced, int n_tokens,
                               int pos0, int32_t* preds, float* hidden, void* scratch,
                               size_t scratch_bytes, void* cuda_stream) {
  cudaStream_t stream = (cudaStream_t)cuda_stream;
  if (!P || !forced || !preds || !scratch || n_forced < 1 || n_tokens < 1 || pos0 < 0 ||
      (long long)pos0 + n_tokens > P->max_pos)
    return LXB_E_INVAL;
  const Layout l = layout(P);
  if (scratch_bytes < l.total || ((uintptr_t)scratch & 255)) return LXB_E_INVAL;
  unsigned char* b = (unsigned char*)scratch;
  cudaError_t e = cudaMemsetAsync(b + l.bar, 0, l.apart - l.bar, stream);
  if (e != cudaSuccess) return (int)e;
  TP p{};
  p.layers = P->d_layers;
  p.n_layers = P->n_layers;
  p.n_vocab = P->n_vocab;
  p.n_embed = P->n_embed;
  p.max_pos = P->max_pos;
  p.n_forced = n_forced;
  p.n_tokens = n_tokens;
  p.pos0 = pos0;
  p.nsplit = P->nsplit;
  p.eps = P->eps;
  p.embed = P->embed;
  p.head = P->head;
  p.fnorm = P->fnorm;
  p.rope = P->rope;
  p.forced = forced;
  p.preds = preds;
  p.hidden = hidden;
  p.bar = (unsigned long long*)(b + l.bar);
  p.abort_flag = (int*)(b + l.bar + 8);
  p.xg = (uint32_t*)(b + l.xg);
  p.proj = (uint32_t*)(b + l.proj);
  p.vec = (uint32_t*)(b + l.vec);
  p.act = (uint32_t*)(b + l.act);
  p.acnt = (unsigned int*)(b + l.bar + 16);
  p.apart = (float*)(b + l.apart);
  p.amax = (float*)(b + l.amax);
  p.aidx = (int*)(b + l.aidx);
  p.status = P->d_status;
  p.prof = P->prof;
  void* args[] = {&p};
  e = cudaLaunchCooperativeKernel((const void*)lxb_text_kernel, dim3(P->grid), dim3(NT), args,
                                  (size_t)P->smem, stream);
  return (int)e;
}

extern "C" int lxb_text_status(lxb_text_plan* P, uint32_t* status) {
  if (!P || !status) return LXB_E_INVAL;
  return (int)cudaMemcpy(status, P->d_status, 4, cudaMemcpyDeviceToHost);
}

extern "C" int lxb_text_status_clear(lxb_text_plan* P) {
  if (!P) return LXB_E_INVAL;
  return (int)cudaMemset(P->d_status, 0, 16);
}

extern "C" int lxb_text_grid(const lxb_text_plan* P) { return P ? P->grid : 0; }

extern "C" int lxb_text_set_profile(lxb_text_plan* P, unsigned long long* prof) {
  if (!P) return LXB_E_INVAL;
  P->prof = prof;
  return 0;
}

extern "C" void lxb_text_plan_destroy(lxb_text_plan* P) {
  if (!P) return;
  if (P->d_layers) cudaFree(P->d_layers);
  if (P->d_status) cudaFree(P->d_status);
  delete P;
}
