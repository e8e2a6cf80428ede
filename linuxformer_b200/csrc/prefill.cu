// linuxformer-b200: the sparse chunked prefill (verified mode) on sm_100a.
//
// The reference checks a proposed token trace as chunked prefill: Session.verify
// (lx/lx/session.py:86-116) runs each chunk through Fast.forward (lx/lx/fast.py:252-361: the
// projections over the live columns, the causal conv, fla's chunk_gated_delta_rule over the active
// (key head, block) pairs, the gated norm and out_proj, the MLP) and Fast.head_argmax
// (fast.py:544-550), and compares each position's argmax with the next token.
//
// Here a chunk of T tokens runs layer by layer, every stage over the whole chunk at once:
//   embed / rows in -> per layer: input norm -> tap-channel projections, gates (beta, exp(g))
//   -> conv + silu -> query/key l2 norms -> recurrence -> gated norm -> out_proj -> post norm
//   -> MLP -> final norm -> head argmax -> first mismatch.
// Activations are kept feature-major ([feature][token], bf16 bits), so a warp's 32 lanes are 32
// consecutive tokens: a weight entry is read once per warp (a uniform load) and its input column
// is one coalesced 64-byte read. Every sum is taken by one thread in the canonical order of the
// CPU restatement (oracle/oracle.c), so the chunk's results are the per-token decode's bits:
// predictions, conv windows and recurrent states.
//
// The recurrence. A key head's query and key can be nonzero only on its live rows (the rows of
// its channels with a nonzero conv tap, at most LXB_PF_MAXLIVE), so each value head's state has
// two parts: the live rows, which the delta rule reads and writes, and the rest, which only
// decays (S <- S * exp(g_t) every token). The live rows of one column sit in one thread's
// registers for the whole chunk (lpf_recur: a CTA per value head, a thread per column, the
// token loop sequential as the recurrence is). The other rows are scaled token by token
// (lpf_scan, one float4 per thread; the same rounding as the per-token decode, so the state is
// bit-identical), on a second stream as soon as the layer's gates exist, and a thread stops as
// soon as its four values are zero (they stay zero). Nothing here waits on another CTA or rank:
// there is no spin and no grid-wide barrier; the stages are ordinary launches.
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <mutex>
#include <new>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

#include "lxb.h"
#include "lxb_math.h"
#include "lxb_prefill.h"

namespace {

constexpr int H = 2560, KD = 256, VD = 128, NK = 16, NV = 128, R = 8, CONV = 24576;
constexpr int TPAD = 256;    // the token dimension of every buffer is padded to this
constexpr int ROWT = 256;    // tokens per block in the row kernels (128 threads, 2 tokens each)
constexpr int HEAD_ROWS = 16384;  // head rows per slice (lpf_head_tile)

__device__ __forceinline__ float bf(uint16_t b) { return lx_f(b); }
__device__ __forceinline__ float bflo(uint32_t u) { return lx_f((uint16_t)(u & 0xffffu)); }
__device__ __forceinline__ float bfhi(uint32_t u) { return lx_f((uint16_t)(u >> 16)); }
__device__ __forceinline__ uint32_t pack2(uint16_t a, uint16_t b) {
  return (uint32_t)a | ((uint32_t)b << 16);
}

// Device view of an uploaded prefill plan.
struct PV {
  const lxb_pf_layer* layers;
  const uint32_t* ent;
  const int32_t* i32;
  const uint16_t* u16;
  const lxb_pf_tap* taps;
  const lxb_pf_vh* vhs;
  const lxb_pf_unit* units;
  const unsigned long long* hcodes;
  uint32_t* status;  // [0] LXB_S_* bits, [1] first stream (0), [2] first token
};

// Scratch buffers of one call (token stride Tp, a multiple of TPAD).
struct Buf {
  int T, Tp;        // tokens of this view; the token stride of every [..][Tp] buffer
  int Te;           // this view's padded extent (a multiple of 256, at most Tp - its offset)
  int t_off;        // this view's first token in the call
  int T_call;       // the call's tokens (the mismatch check runs up to the call's end)
  int os;           // the token stride of o (max live value heads x 128)
  uint16_t* x;      // [H][Tp] residual (bf16 values)
  uint16_t* xn;     // [H][Tp] the current norm's output
  uint16_t* P;      // [max_tap][Tp] tap channels' projections
  uint16_t* Y;      // [max_tap][Tp] tap channels' conv + silu
  float* e;         // [n_layers][NV][Tp] exp(g) (1 where g = 0)
  float* beta;      // [NV][Tp]
  float* qs;        // [max_slot][Tp] query l2norm * 0.0625 on live rows
  float* ks;        // [max_slot][Tp] key l2norm on live rows
  uint32_t* qm;     // [NK][Tp] bit s: slot s's query is nonzero; bit 31: any raw query nonzero
  uint32_t* km;     // [NK][Tp] the same for keys
  uint16_t* o;      // [Tp][max_lvh * VD] the recurrence's output (token-major)
  uint16_t* on;     // [max_lvh * VD][Tp] gated-norm output
  uint16_t* hb;     // [max_units][Tp] MLP activations
  uint2* hp;        // [n_slices][Tp] head partial maxima (value bits, row)
  uint32_t* flags;  // [n_layers][NV]: some exp(g) != 1 in this view
  int* fw;          // the first mismatch (working value)
};

// --- rows in / out: [T][H] bf16 rows <-> [H][Tp] ----------------------------------------------
// src row of token t: tok ? offset + tok[t] : t. A token id outside the embedding is clamped to
// row offset and reported (LXB_S_TOKEN with its position).
__global__ void __launch_bounds__(256) lpf_rows_in(const uint16_t* src, const int32_t* tok,
                                                   int offset, long long n_rows, int T, int Tp,
                                                   uint16_t* x, uint32_t* status) {
  __shared__ uint16_t tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int k = ty; k < 32; k += 8) {
    const int t = t0 + k;
    uint16_t v = 0;
    if (t < T) {
      long long row = t;
      if (tok) {
        long long id = tok[t];
        if (id < 0 || id + offset >= n_rows) {
          if (tx == 0 && blockIdx.y == 0 && atomicOr(status, LXB_S_TOKEN) == 0) {
            status[1] = 0;
            status[2] = (uint32_t)t;
          }
          id = 0;
        }
        row = id + offset;
      }
      v = src[row * H + c0 + tx];
    }
    tile[k][tx] = v;
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) x[(size_t)(c0 + k) * Tp + t0 + tx] = tile[tx][k];
}

__global__ void __launch_bounds__(256) lpf_rows_out(const uint16_t* x, int T, int Tp,
                                                    uint16_t* dst) {
  __shared__ uint16_t tile[32][33];
  const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int k = ty; k < 32; k += 8) tile[k][tx] = x[(size_t)(c0 + k) * Tp + t0 + tx];
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    const int t = t0 + k;
    if (t < T) dst[(size_t)t * H + c0 + tx] = tile[tx][k];
  }
}

// --- Qwen3_5RMSNorm per token ------------------------------------------------------------------
// The canonical 2560-element sum of squares (lane l of 512 sums x[l + 512 i]^2, i = 0..4; an xor
// butterfly over each 32 lanes; one over the 16 partial sums), taken by one thread per token; then
// xn = bf16(x * rsqrt(ssq / 2560 + eps) * (1 + w)).
// A block takes 32 tokens (lane = token) with 16 warps: warp g sums the canonical lanes
// 32 g .. 32 g + 31 of its token (each 5 squares, then that group's butterfly) in one thread,
// warp 0 folds the 16 group sums, and all 512 threads write the normed columns.
__global__ void __launch_bounds__(512) lpf_norm(const uint16_t* __restrict__ x, int T, int Tp,
                                                const uint16_t* __restrict__ w, float eps,
                                                uint16_t* __restrict__ xn) {
  __shared__ float s_w[16][32];
  __shared__ float s_r[32];
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int t0 = blockIdx.x * 32, t = t0 + lane;
  const uint16_t* xc = x + t;  // (t < Tp: the buffers are padded; tokens past T are not used)
  float v[32];
#pragma unroll
  for (int l = 0; l < 32; l++) {
    const int c = g * 32 + l;
    float a = bf(xc[(size_t)c * Tp]);
    float sq = lx_mul(a, a);
#pragma unroll
    for (int i = 1; i < 5; i++) {
      a = bf(xc[(size_t)(c + 512 * i) * Tp]);
      sq = lx_add(sq, lx_mul(a, a));
    }
    v[l] = sq;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int l = 0; l < off; l++) v[l] = lx_add(v[l], v[l + off]);
  s_w[g][lane] = v[0];
  __syncthreads();
  if (g == 0) {
    float ws[16];
#pragma unroll
    for (int k = 0; k < 16; k++) ws[k] = s_w[k][lane];
#pragma unroll
    for (int off = 8; off > 0; off >>= 1)
#pragma unroll
      for (int k = 0; k < off; k++) ws[k] = lx_add(ws[k], ws[k + off]);
    s_r[lane] = lx_rsqrt(lx_add(lx_div(ws[0], (float)H), eps));
  }
  __syncthreads();
  if (t >= T) return;
  const float r = s_r[lane];
#pragma unroll 4
  for (int c = g; c < H; c += 16) {
    const float w1 = lx_add(1.0f, bf(__ldg(w + c)));
    xn[(size_t)c * Tp + t] = lx_rb(lx_mul(lx_mul(bf(xc[(size_t)c * Tp]), r), w1));
  }
}

// Sequential sums over a row's entries (index | bf16 << 16) for two consecutive tokens, from +0:
// up to DW entries at a time, their input columns read at once (the loads first, then the adds
// in order), so a row costs one or two memory round trips instead of one per entry.
constexpr int DW = 4;
struct Acc2 {
  float a0 = 0.0f, a1 = 0.0f;
};
template <bool SKIP_ZERO>
__device__ __forceinline__ void acc2(Acc2& a, bool& any0, bool& any1, uint32_t e, uint32_t xx) {
  const float w = bfhi(e);
  const float v0 = bflo(xx), v1 = bfhi(xx);
  if (!SKIP_ZERO || v0 != 0.0f) {
    a.a0 = lx_add(a.a0, lx_mul(v0, w));
    any0 = true;
  }
  if (!SKIP_ZERO || v1 != 0.0f) {
    a.a1 = lx_add(a.a1, lx_mul(v1, w));
    any1 = true;
  }
}
// NR rows (row r: entries ep[r][0..n[r])), their sums advancing together
template <int NR, bool SKIP_ZERO>
__device__ __forceinline__ void dotsn(const uint32_t* const* __restrict__ ep, const uint32_t* n,
                                      const uint16_t* __restrict__ x, int Tp, int t, Acc2* acc,
                                      bool* any) {
  const uint16_t* xt = x + t;
  uint32_t nmax = n[0];
#pragma unroll
  for (int r = 1; r < NR; r++) nmax = max(nmax, n[r]);
  for (uint32_t k = 0; k < nmax; k += DW) {
    uint32_t e[NR][DW], xx[NR][DW];
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
      for (int q = 0; q < DW; q++) e[r][q] = k + q < n[r] ? __ldg(ep[r] + k + q) : 0u;
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
      for (int q = 0; q < DW; q++)
        xx[r][q] = k + q < n[r] ? *reinterpret_cast<const uint32_t*>(
                                      xt + (size_t)(e[r][q] & 0xffffu) * Tp)
                                : 0u;
#pragma unroll
    for (int r = 0; r < NR; r++)
#pragma unroll
      for (int q = 0; q < DW; q++)
        if (k + q < n[r]) acc2<SKIP_ZERO>(acc[r], any[2 * r], any[2 * r + 1], e[r][q], xx[r][q]);
  }
}
template <int NR, bool SKIP_ZERO>
__device__ __forceinline__ void dots(const uint32_t* __restrict__ e0p, uint32_t n0,
                                     const uint32_t* __restrict__ e1p, uint32_t n1,
                                     const uint16_t* __restrict__ x, int Tp, int t, Acc2* acc,
                                     bool* any) {
  const uint32_t* ep[2] = {e0p, e1p};
  const uint32_t n[2] = {n0, n1};
  dotsn<NR, SKIP_ZERO>(ep, n, x, Tp, t, acc, any);
}

__device__ __forceinline__ void dot2(const uint32_t* __restrict__ ent, uint32_t n,
                                     const uint16_t* __restrict__ xn, int Tp, int t, float& a0,
                                     float& a1) {
  Acc2 acc[1];
  bool any[2] = {false, false};
  dots<1, false>(ent, n, nullptr, 0, xn, Tp, t, acc, any);
  a0 = acc[0].a0;
  a1 = acc[0].a1;
}

// tap channels' in_proj_qkv projections: P = bf16(row . xn)
__global__ void __launch_bounds__(128) lpf_taps(PV pv, int tap0, Buf b) {
  const int t = blockIdx.x * ROWT + 2 * threadIdx.x;
  const lxb_pf_tap tp = pv.taps[tap0 + blockIdx.y];
  float a0, a1;
  dot2(pv.ent + tp.ent, tp.n, b.xn, b.Tp, t, a0, a1);
  *reinterpret_cast<uint32_t*>(b.P + (size_t)blockIdx.y * b.Tp + t) =
      pack2(lx_rb(a0), lx_rb(a1));
}

// beta = bf16(sigmoid(bf16(b . xn))); g = -exp(A_log) * softplus(bf16(a . xn) + dt_bias);
// e = exp(g), or 1 where g = 0 (a multiplication by 1 leaves every value as it is)
__global__ void __launch_bounds__(128) lpf_gates(PV pv, int L, Buf b) {
  const int vh = blockIdx.y;
  const int t = blockIdx.x * ROWT + 2 * threadIdx.x;
  const lxb_pf_vh p = pv.vhs[(size_t)L * NV + vh];
  Acc2 ab[2];
  bool any[4] = {false, false, false, false};
  dots<2, false>(pv.ent + p.a_ent, p.a_n, pv.ent + p.b_ent, p.b_n, b.xn, b.Tp, t, ab, any);
  const float a[2] = {ab[0].a0, ab[0].a1}, bb[2] = {ab[1].a0, ab[1].a1};
  const float A = -lx_exp(bf(p.A_log));
  const float dt = bf(p.dt_bias);
  float ev[2], be[2];
  bool dec = false;
#pragma unroll
  for (int k = 0; k < 2; k++) {
    be[k] = lx_rbf(lx_sigmoid(lx_rbf(bb[k])));
    const float g = lx_mul(A, lx_softplus(lx_add(lx_rbf(a[k]), dt)));
    ev[k] = g != 0.0f ? lx_exp(g) : 1.0f;
    dec |= (t + k < b.T) && ev[k] != 1.0f;
  }
  float* e = b.e + ((size_t)L * NV + vh) * b.Tp;
  *reinterpret_cast<float2*>(e + t) = make_float2(ev[0], ev[1]);
  *reinterpret_cast<float2*>(b.beta + (size_t)vh * b.Tp + t) = make_float2(be[0], be[1]);
  if (__syncthreads_or(dec) && threadIdx.x == 0) atomicOr(b.flags + (size_t)L * NV + vh, 1u);
}

// conv + silu of the tap channels: y_t = k0 P(t-3) + k1 P(t-2) + k2 P(t-1) + k3 P(t) from +0, the
// P before the chunk from the channel's conv window; Y = bf16(silu(bf16(y)))
__global__ void __launch_bounds__(128) lpf_conv(PV pv, int tap0, const uint64_t* __restrict__ sp,
                                                int L, Buf b) {
  const uint16_t* conv = reinterpret_cast<const uint16_t*>(sp[2 * L + 1]);
  const int t = blockIdx.x * ROWT + 2 * threadIdx.x;
  const lxb_pf_tap tp = pv.taps[tap0 + blockIdx.y];
  const uint16_t* Pr = b.P + (size_t)blockIdx.y * b.Tp;
  const uint16_t* w = conv + (size_t)tp.conv_ch * 4;
  const float k0 = bflo(tp.t01), k1 = bfhi(tp.t01), k2 = bflo(tp.t23), k3 = bfhi(tp.t23);
  uint16_t out[2];
#pragma unroll
  for (int k = 0; k < 2; k++) {
    const int u = t + k;
    auto at = [&](int v) -> float { return bf(v >= 0 ? Pr[v] : w[4 + v]); };
    float y = 0.0f;
    y = lx_add(y, lx_mul(k0, at(u - 3)));
    y = lx_add(y, lx_mul(k1, at(u - 2)));
    y = lx_add(y, lx_mul(k2, at(u - 1)));
    y = lx_add(y, lx_mul(k3, at(u)));
    out[k] = lx_rb(lx_silu(lx_rbf(y)));
  }
  *reinterpret_cast<uint32_t*>(b.Y + (size_t)blockIdx.y * b.Tp + t) = pack2(out[0], out[1]);
}

// The conv windows the chunk leaves: [P(T-4), .., P(T-1)] (the old window's tail first when
// T < 4). A channel without in_proj_qkv entries gets P = +0 only while its window holds a
// nonzero value; once the window is all zeros the per-token decode leaves it as it is.
__global__ void __launch_bounds__(128) lpf_windows(PV pv, const lxb_pf_layer* lyp,
                                                   const uint64_t* __restrict__ sp, int L, Buf b) {
  const int ch = blockIdx.x * 128 + threadIdx.x;
  if (ch >= CONV) return;
  uint16_t* conv = reinterpret_cast<uint16_t*>(sp[2 * L + 1]);
  const lxb_pf_layer ly = *lyp;
  const int32_t* c = pv.i32 + ly.chan + 3 * ch;
  const int tap = c[0], off = c[1], n = c[2];
  uint16_t* w = conv + (size_t)ch * 4;
  uint16_t nw[4] = {w[0], w[1], w[2], w[3]};
  if (n == 0) {  // P = +0 every step: shift zeros in while the window is not all zero
    for (int s = 0; s < 4 && s < b.T; s++) {
      if (((nw[0] | nw[1] | nw[2] | nw[3]) & 0x7fff) == 0) break;
      nw[0] = nw[1];
      nw[1] = nw[2];
      nw[2] = nw[3];
      nw[3] = 0;
    }
  } else {
    for (int k = 0; k < 4; k++) {
      const int u = b.T - 4 + k;
      if (u < 0) {
        nw[k] = w[4 + u];
      } else if (tap >= 0) {
        nw[k] = b.P[(size_t)tap * b.Tp + u];
      } else {
        float s = 0.0f;
        for (int q = 0; q < n; q++) {
          const uint32_t e = pv.ent[off + q];
          s = lx_add(s, lx_mul(bf(b.xn[(size_t)(e & 0xffffu) * b.Tp + u]), bfhi(e)));
        }
        nw[k] = lx_rb(s);
      }
    }
  }
  *reinterpret_cast<uint2*>(w) = make_uint2(pack2(nw[0], nw[1]), pack2(nw[2], nw[3]));
}

// The live key heads' query and key l2 norms (transformers' l2norm in bf16: x * rsqrt(sum of the
// nonzero bf16 squares, ascending + 1e-6)), on the live rows only: every other row is +0.
__global__ void __launch_bounds__(128) lpf_qk(PV pv, const lxb_pf_layer* lyp, Buf b) {
  const int t = blockIdx.x * 128 + threadIdx.x;
  if (t >= b.T) return;
  const lxb_pf_layer ly = *lyp;
  const int32_t* kh = pv.i32 + ly.khs + 3 * blockIdx.y;
  const int s0 = kh[1], nl = kh[2];
  const int32_t* sl = pv.i32 + ly.slots + 3 * s0;
#pragma unroll
  for (int which = 0; which < 2; which++) {  // 0 query, 1 key
    bool any = false;
    float ss = 0.0f;
    for (int s = 0; s < nl; s++) {
      const int tp = sl[3 * s + 1 + which];
      const float v = tp >= 0 ? bf(b.Y[(size_t)tp * b.Tp + t]) : 0.0f;
      any |= v != 0.0f;
      const float sq = lx_rbf(lx_mul(v, v));
      if (sq != 0.0f) ss = lx_add(ss, sq);
    }
    uint32_t mask = any ? 0x80000000u : 0u;
    float inv = 0.0f;
    if (any) {
      const float se = lx_rbf(lx_add(lx_rbf(ss), 1e-6f));
      inv = lx_rbf(lx_rsqrt(se));
    }
    float* dst = (which ? b.ks : b.qs) + (size_t)s0 * b.Tp + t;
    for (int s = 0; s < nl; s++) {
      float out = 0.0f;
      if (any) {
        const int tp = sl[3 * s + 1 + which];
        const float v = tp >= 0 ? bf(b.Y[(size_t)tp * b.Tp + t]) : 0.0f;
        const float n = lx_rbf(lx_mul(v, inv));
        if (n != 0.0f) mask |= 1u << s;
        out = which ? n : lx_mul(n, 0.0625f);
      }
      dst[(size_t)s * b.Tp] = out;
    }
    (which ? b.km : b.qm)[(size_t)blockIdx.y * b.Tp + t] = mask;
  }
}

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The recurrence over the live rows of one value head (a CTA per live value head, a thread per
// column j; NL register slots, the key head's live rows in ascending order). Per token, as the
// per-token decode: S *= exp(g); if a key: kv = sum over the key's nonzero rows S k, delta =
// (v - kv) beta, S += k delta; if a query: o = bf16(sum over the query's nonzero rows S q/16).
// The body has no branch: a slot whose key or query value is zero (a zero row, a token without
// a key or query, a slot past the head's live rows) adds S * 0 = +-0 to a sum that started at +0,
// which leaves the sum's bits as they are (+0 + -0 = +0; x + +-0 = x for x != 0); the state
// itself takes k delta only where the key's mask bit is set (a select: a -0 state value keeps its
// sign). So the tokens of a tile form one basic block and the compiler overlaps a token's loads
// with the previous token's chain.
// The per-token inputs shared by the CTA (exp(g), beta, the key mask, the live rows' query and
// key values) come through shared memory in double-buffered tiles of RT tokens (cp.async, the
// next tile in flight while this one runs); each thread's value column for the tile sits in
// registers (prefetched a tile ahead).
constexpr int RT = 32;  // tokens per recurrence tile
template <int NL>
__device__ __forceinline__ void recur_token(float (&S)[NL], const float4 tk, const float* kp,
                                            const float* qp, float v, uint16_t* out) {
  constexpr int NP = (NL + 3) / 4 * 4;
  float kk[NP], qq[NP];
#pragma unroll
  for (int s = 0; s < NP; s += 4) {
    const float4 a = *reinterpret_cast<const float4*>(kp + s);
    const float4 c = *reinterpret_cast<const float4*>(qp + s);
    kk[s] = a.x, kk[s + 1] = a.y, kk[s + 2] = a.z, kk[s + 3] = a.w;
    qq[s] = c.x, qq[s + 1] = c.y, qq[s + 2] = c.z, qq[s + 3] = c.w;
  }
  const uint32_t km = __float_as_uint(tk.z);
#pragma unroll
  for (int s = 0; s < NL; s++) S[s] = lx_mul(S[s], tk.x);
  float kv = 0.0f;
#pragma unroll
  for (int s = 0; s < NL; s++) kv = lx_add(kv, lx_mul(S[s], kk[s]));
  const float delta = lx_mul(lx_sub(v, kv), tk.y);
#pragma unroll
  for (int s = 0; s < NL; s++) {
    const float nv = lx_add(S[s], lx_mul(kk[s], delta));
    S[s] = ((km >> s) & 1u) ? nv : S[s];
  }
  float o = 0.0f;
#pragma unroll
  for (int s = 0; s < NL; s++) o = lx_add(o, lx_mul(S[s], qq[s]));
  *out = lx_rb(o);
}

template <int NL>
__global__ void __launch_bounds__(128) lpf_recur(PV pv, const lxb_pf_layer* lyp, int L,
                                                 const uint64_t* __restrict__ sp, Buf b) {
  constexpr int NP = (NL + 3) / 4 * 4;
  __shared__ __align__(16) float4 s_tok[2][RT];      // exp(g), beta, key mask, query mask
  __shared__ __align__(16) float s_k[2][RT][NP];
  __shared__ __align__(16) float s_q[2][RT][NP];
  const lxb_pf_layer ly = *lyp;
  const int lvh = blockIdx.x, i = lvh / R, r = lvh % R;
  const int j = threadIdx.x;
  const int32_t* khp = pv.i32 + ly.khs + 3 * i;
  const int kh = khp[0], s0 = khp[1], nl = khp[2];
  const int vh = kh * R + r;
  const int32_t* sl = pv.i32 + ly.slots + 3 * s0;
  float* rec = reinterpret_cast<float*>(sp[2 * L]);
  float* Sg = rec + (size_t)vh * KD * VD + j;
  float S[NL];
#pragma unroll
  for (int s = 0; s < NL; s++) S[s] = s < nl ? Sg[(size_t)sl[3 * s] * VD] : 0.0f;
  const int vt = pv.i32[ly.vtap + lvh * VD + j];
  const float* ev = b.e + ((size_t)L * NV + vh) * b.Tp;
  const float* bv = b.beta + (size_t)vh * b.Tp;
  const uint32_t* qmv = b.qm + (size_t)i * b.Tp;
  const uint32_t* kmv = b.km + (size_t)i * b.Tp;
  const float* ksv = b.ks + (size_t)s0 * b.Tp;
  const float* qsv = b.qs + (size_t)s0 * b.Tp;
  const uint4* vsrc = vt >= 0 ? reinterpret_cast<const uint4*>(b.Y + (size_t)vt * b.Tp) : nullptr;
  const int ostride = b.os;
  uint16_t* op = b.o + lvh * VD + j;
  // the slots past the head's live rows stay zero in both buffers (nothing copies into them)
  for (int k = j; k < 2 * RT * NP; k += 128) {
    const int s = k % NP;
    if (s >= nl) {
      (&s_k[0][0][0])[k] = 0.0f;
      (&s_q[0][0][0])[k] = 0.0f;
    }
  }
  auto issue = [&](int buf, int t0) {
    for (int k = j; k < RT * 4; k += 128) {
      const int tt = k >> 2, f = k & 3;
      const void* src = f == 0 ? (const void*)(ev + t0 + tt) : f == 1 ? (const void*)(bv + t0 + tt)
                        : f == 2 ? (const void*)(kmv + t0 + tt) : (const void*)(qmv + t0 + tt);
      cp_async4(reinterpret_cast<float*>(&s_tok[buf][tt]) + f, src);
    }
    for (int k = j; k < RT * nl; k += 128) {
      const int s = k / RT, tt = k % RT;
      cp_async4(&s_k[buf][tt][s], ksv + (size_t)s * b.Tp + t0 + tt);
      cp_async4(&s_q[buf][tt][s], qsv + (size_t)s * b.Tp + t0 + tt);
    }
    cp_commit();
  };
  uint4 vc[RT / 8], vn[RT / 8];  // this tile's and the next tile's value column (bf16 pairs)
#pragma unroll
  for (int q = 0; q < RT / 8; q++) vc[q] = vsrc ? vsrc[q] : make_uint4(0, 0, 0, 0);
  issue(0, 0);
  int buf = 0;
  for (int t0 = 0; t0 < b.T; t0 += RT) {
    const bool more = t0 + RT < b.T;
    if (more) {
      issue(buf ^ 1, t0 + RT);
#pragma unroll
      for (int q = 0; q < RT / 8; q++)
        vn[q] = vsrc ? vsrc[(t0 + RT) / 8 + q] : make_uint4(0, 0, 0, 0);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    uint16_t* ot = op + (size_t)t0 * ostride;
    if (b.T - t0 >= RT) {  // a whole tile: one basic block
#pragma unroll
      for (int tt = 0; tt < RT; tt++) {
        const uint32_t vw = (&vc[tt / 8].x)[(tt % 8) / 2];
        recur_token<NL>(S, s_tok[buf][tt], s_k[buf][tt], s_q[buf][tt],
                        (tt & 1) ? bfhi(vw) : bflo(vw), ot + (size_t)tt * ostride);
      }
    } else {
      const int n = b.T - t0;
#pragma unroll
      for (int tt = 0; tt < RT; tt++) {
        if (tt < n) {
          const uint32_t vw = (&vc[tt / 8].x)[(tt % 8) / 2];
          recur_token<NL>(S, s_tok[buf][tt], s_k[buf][tt], s_q[buf][tt],
                          (tt & 1) ? bfhi(vw) : bflo(vw), ot + (size_t)tt * ostride);
        }
      }
    }
    __syncthreads();  // the buffer is reused by the issue two tiles on
#pragma unroll
    for (int q = 0; q < RT / 8; q++) vc[q] = vn[q];
    buf ^= 1;
  }
#pragma unroll
  for (int s = 0; s < NL; s++)
    if (s < nl) Sg[(size_t)sl[3 * s] * VD] = S[s];
}

// The decay of every other state row: S <- S * exp(g_t), token by token (the per-token decode's
// rounding), a float4 per thread (a block: 8 rows of one value head); the factors come through
// shared memory in double-buffered tiles. A thread is done once its four values are zero (they
// stay zero); the block stops when all its threads are.
constexpr int ST = 1024;  // tokens per scan tile
__global__ void __launch_bounds__(256) lpf_scan(PV pv, const lxb_pf_layer* lyp, int L,
                                                const uint64_t* __restrict__ sp, Buf b) {
  __shared__ __align__(16) float s_e[2][ST];
  const int vh = blockIdx.x;
  const int row = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int c4 = threadIdx.x & 31;
  if (!b.flags[(size_t)L * NV + vh]) return;
  const lxb_pf_layer ly = *lyp;
  const uint32_t live = (uint32_t)pv.i32[ly.livemask + (vh / R) * 8 + row / 32];
  float* rec = reinterpret_cast<float*>(sp[2 * L]);
  float4* p = reinterpret_cast<float4*>(rec + ((size_t)vh * KD + row) * VD) + c4;
  float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  bool act = !((live >> (row % 32)) & 1u);
  if (act) {
    v = *p;
    act = v.x != 0.0f || v.y != 0.0f || v.z != 0.0f || v.w != 0.0f;
  }
  const bool wrote = act;
  if (!__syncthreads_or(act)) return;
  const float* ev = b.e + ((size_t)L * NV + vh) * b.Tp;
  auto issue = [&](int buf, int t0) {  // b.Te is a multiple of 256: reads stay inside the view
    for (int k = threadIdx.x; k < ST / 4 && t0 + 4 * k < b.Te; k += 256)
      cp_async16(&s_e[buf][4 * k], ev + t0 + 4 * k);
    cp_commit();
  };
  issue(0, 0);
  int buf = 0;
  for (int t0 = 0; t0 < b.T; t0 += ST) {
    if (t0 + ST < b.T) {
      issue(buf ^ 1, t0 + ST);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (act) {
      const int n = min(ST, b.T - t0);
      const float4* e4 = reinterpret_cast<const float4*>(s_e[buf]);
      int tt = 0;
      for (; tt + 4 <= n; tt += 4) {
        const float4 e = e4[tt / 4];
        v.x = lx_mul(lx_mul(lx_mul(lx_mul(v.x, e.x), e.y), e.z), e.w);
        v.y = lx_mul(lx_mul(lx_mul(lx_mul(v.y, e.x), e.y), e.z), e.w);
        v.z = lx_mul(lx_mul(lx_mul(lx_mul(v.z, e.x), e.y), e.z), e.w);
        v.w = lx_mul(lx_mul(lx_mul(lx_mul(v.w, e.x), e.y), e.z), e.w);
      }
      for (; tt < n; tt++) {
        const float e = s_e[buf][tt];
        v.x = lx_mul(v.x, e);
        v.y = lx_mul(v.y, e);
        v.z = lx_mul(v.z, e);
        v.w = lx_mul(v.w, e);
      }
      act = v.x != 0.0f || v.y != 0.0f || v.z != 0.0f || v.w != 0.0f;
    }
    if (!__syncthreads_or(act)) break;  // also: no thread still reads buf when it is refilled
    buf ^= 1;
  }
  cp_wait<0>();
  if (wrote) *p = v;
}

// Qwen3_5RMSNormGated per (token, live value head): bf16(bf16(w bf16(o rsqrt(mean(o^2) + eps)))
// silu(bf16(z . xn))), the sum of squares as lane l of 32 summing o[4l..4l+3]^2 then an xor
// butterfly; a head whose 128 outputs are all zero gives zeros (the decode skips it). Two tokens
// per thread; the in_proj_z rows four at a time.
__device__ __forceinline__ float o_rr(const uint16_t* orow, float eps, bool& nz) {
  float v[32];
  nz = false;
#pragma unroll
  for (int l = 0; l < 32; l++) {
    const uint2 u = *reinterpret_cast<const uint2*>(orow + 4 * l);
    const float a = bflo(u.x), c = bfhi(u.x), d = bflo(u.y), f = bfhi(u.y);
    nz |= a != 0.0f || c != 0.0f || d != 0.0f || f != 0.0f;
    float s = lx_mul(a, a);
    s = lx_add(s, lx_mul(c, c));
    s = lx_add(s, lx_mul(d, d));
    s = lx_add(s, lx_mul(f, f));
    v[l] = s;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1)
#pragma unroll
    for (int l = 0; l < off; l++) v[l] = lx_add(v[l], v[l + off]);
  return lx_rsqrt(lx_add(lx_div(v[0], 128.0f), eps));
}

__global__ void __launch_bounds__(128) lpf_gnorm(PV pv, const lxb_pf_layer* lyp, float eps,
                                                 Buf b) {
  const int t = blockIdx.y * ROWT + 2 * threadIdx.x;  // heads vary fastest (xn stays in L2)
  if (t >= b.T) return;
  const lxb_pf_layer ly = *lyp;
  const int lvh = blockIdx.x;
  const int ostride = b.os;
  const uint16_t* o0 = b.o + (size_t)t * ostride + lvh * VD;
  const uint16_t* o1 = o0 + ostride;  // token t + 1 (inside the padded buffer)
  uint32_t* on = reinterpret_cast<uint32_t*>(b.on + (size_t)lvh * VD * b.Tp + t);
  bool nz0, nz1;
  const float r0 = o_rr(o0, eps, nz0);
  const float r1 = o_rr(o1, eps, nz1);
  nz1 = nz1 && t + 1 < b.T;
  if (!nz0 && !nz1) {
    for (int k = 0; k < VD; k++) on[(size_t)k * b.Tp / 2] = 0u;
    return;
  }
  const uint16_t* gw = pv.u16 + ly.gnorm;
  const int32_t* zr = pv.i32 + ly.zrow + 2 * lvh * VD;
  for (int k0 = 0; k0 < VD; k0 += 4) {
    const uint32_t* ep[4];
    uint32_t n[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      ep[q] = pv.ent + __ldg(zr + 2 * (k0 + q));
      n[q] = (uint32_t)__ldg(zr + 2 * (k0 + q) + 1);
    }
    Acc2 z[4];
    bool any[8];
    dotsn<4, false>(ep, n, b.xn, b.Tp, t, z, any);
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const int k = k0 + q;
      const float w = bf(__ldg(gw + k));
      uint16_t h0 = 0, h1 = 0;
      if (nz0) {
        const float u = lx_rbf(lx_mul(w, lx_rbf(lx_mul(bf(o0[k]), r0))));
        h0 = lx_rb(lx_mul(u, lx_silu(lx_rbf(z[q].a0))));
      }
      if (nz1) {
        const float u = lx_rbf(lx_mul(w, lx_rbf(lx_mul(bf(o1[k]), r1))));
        h1 = lx_rb(lx_mul(u, lx_silu(lx_rbf(z[q].a1))));
      }
      on[(size_t)k * b.Tp / 2] = pack2(h0, h1);
    }
  }
}

// A residual row's update from a sparse row over an input (out_proj over the gated-norm outputs,
// down_proj over the MLP activations): s = the sum over entries with a nonzero input, in order
// from +0; where any, x = bf16(x + bf16(s)).
__global__ void __launch_bounds__(128) lpf_add_rows(PV pv, int ptr_off,
                                                    const uint16_t* __restrict__ in, Buf b) {
  const int rr = blockIdx.x;  // rows vary fastest: one token block's inputs stay in L2
  const int p0 = pv.i32[ptr_off + rr], p1 = pv.i32[ptr_off + rr + 1];
  if (p0 == p1) return;
  const int t = blockIdx.y * ROWT + 2 * threadIdx.x;
  Acc2 acc[1];
  bool any[2] = {false, false};
  dots<1, true>(pv.ent + p0, (uint32_t)(p1 - p0), nullptr, 0, in, b.Tp, t, acc, any);
  const float s0 = acc[0].a0, s1 = acc[0].a1;
  const bool a0 = any[0], a1 = any[1];
  if (!a0 && !a1) return;
  uint32_t* xp = reinterpret_cast<uint32_t*>(b.x + (size_t)rr * b.Tp + t);
  const uint32_t xx = *xp;
  uint16_t n0 = (uint16_t)(xx & 0xffffu), n1 = (uint16_t)(xx >> 16);
  if (a0) n0 = lx_rb(lx_add(bf(n0), lx_rbf(s0)));
  if (a1) n1 = lx_rb(lx_add(bf(n1), lx_rbf(s1)));
  *xp = pack2(n0, n1);
}

// --- stages over a shared-memory token tile ---------------------------------------------------
// A block takes XT = 32 consecutive tokens and copies their whole normed input ([2560][32] bf16,
// 160 KB) into shared memory; lane l of every warp is token t0 + l, and the warps share out the
// rows (MLP units, head rows). A row's entries are uniform loads (one per warp), its inputs
// conflict-free shared loads (two lanes per 32-bit word), so no input read waits on L2.
constexpr int XT = 32;
constexpr int XW = 16;  // warps per tile block
constexpr int XSMEM = H * XT * 2;

__device__ __forceinline__ void fill_tile(uint16_t* xs, const uint16_t* __restrict__ xn, int Tp,
                                          int t0) {
  for (int k = threadIdx.x; k < H * (XT / 8); k += XW * 32) {
    const int c = k / (XT / 8), q = k % (XT / 8);
    cp_async16(xs + c * XT + q * 8, xn + (size_t)c * Tp + t0 + q * 8);
  }
  cp_commit();
  cp_wait<0>();
  __syncthreads();
}

// Two units' gate and up sums over the tile (lane = token): a unit's gate entries then its up
// entries are one list in the plan; both units' lists walked together four entries at a time
// (the eight loads first, then the adds in order, each into its own sum).
struct UnitSums {
  float g, u;
};
__device__ __forceinline__ void gate_up2(const uint32_t* const* __restrict__ ge,
                                         const uint32_t* ng, const uint32_t* nn,
                                         const uint16_t* xs, int lane, UnitSums* out) {
  out[0] = out[1] = UnitSums{0.0f, 0.0f};
  const uint32_t n = max(nn[0], nn[1]);
  for (uint32_t k = 0; k < n; k += 4) {
    uint32_t e[2][4];
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
      for (int q = 0; q < 4; q++) e[r][q] = k + q < nn[r] ? __ldg(ge[r] + k + q) : 0u;
    float x[2][4];
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
      for (int q = 0; q < 4; q++) x[r][q] = bf(xs[(e[r][q] & 0xffffu) * XT + lane]);
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint32_t i = k + q;
        const float pr = lx_mul(x[r][q], bfhi(e[r][q]));
        if (i < ng[r]) out[r].g = lx_add(out[r].g, pr);
        else if (i < nn[r]) out[r].u = lx_add(out[r].u, pr);
      }
  }
}

// MLP units over a tile: h = bf16(bf16(silu(bf16(gate . xn))) * bf16(up . xn)); each warp takes
// two units at a time and fetches the next pair's descriptors while this pair runs
__global__ void __launch_bounds__(XW * 32) lpf_mlp_tile(PV pv, int unit0, int n_units, Buf b) {
  extern __shared__ __align__(16) uint16_t xs[];
  const int t0 = blockIdx.x * XT;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const lxb_pf_unit* units = pv.units + unit0;
  auto unit = [&](int u) { return u < n_units ? units[u] : lxb_pf_unit{0, 0, 0, 0}; };
  lxb_pf_unit A = unit(warp), B = unit(warp + XW);
  fill_tile(xs, b.xn, b.Tp, t0);
  uint16_t* hb = b.hb + t0 + lane;
  for (int u = warp; u < n_units; u += 2 * XW) {
    const lxb_pf_unit nA = unit(u + 2 * XW), nB = unit(u + 3 * XW);
    const uint32_t* ge[2] = {pv.ent + A.g, pv.ent + B.g};
    const uint32_t ng[2] = {A.ng, B.ng}, nn[2] = {A.ng + A.nu, B.ng + B.nu};
    UnitSums d[2];
    gate_up2(ge, ng, nn, xs, lane, d);
    hb[(size_t)u * b.Tp] = lx_rb(lx_mul(lx_rbf(lx_silu(lx_rbf(d[0].g))), lx_rbf(d[0].u)));
    if (u + XW < n_units)
      hb[(size_t)(u + XW) * b.Tp] =
          lx_rb(lx_mul(lx_rbf(lx_silu(lx_rbf(d[1].g))), lx_rbf(d[1].u)));
    A = nA;
    B = nB;
  }
}

// a row's dot over the tile (lane = token), four entries at a time
__device__ __forceinline__ float tdot(const uint32_t* __restrict__ ent, uint32_t n,
                                      const uint16_t* xs, int lane) {
  float a = 0.0f;
  for (uint32_t k = 0; k < n; k += 4) {
    uint32_t e[4];
#pragma unroll
    for (int q = 0; q < 4; q++) e[q] = k + q < n ? __ldg(ent + k + q) : 0u;
    float x[4];
#pragma unroll
    for (int q = 0; q < 4; q++) x[q] = bf(xs[(e[q] & 0xffffu) * XT + lane]);
#pragma unroll
    for (int q = 0; q < 4; q++)
      if (k + q < n) a = lx_add(a, lx_mul(x[q], bfhi(e[q])));
  }
  return a;
}

struct HeadArgs {
  int V, n_dense, head_ptr;
  float htab[4];
  int dense_cols[LXB_PF_MAXDENSE];
};

// The head's logit of one row: bf16(D + S), D the dense columns in groups of 4 (each from +0,
// the groups summed in order from +0), S the other entries in order; the prediction is the first
// maximum (a later equal logit does not replace it).
__device__ __forceinline__ float head_dense(const HeadArgs& ha, unsigned long long codes,
                                            const float* xd) {
  float D = 0.0f, grp = 0.0f;
  int in = 0;
#pragma unroll
  for (int j = 0; j < LXB_PF_MAXDENSE; j++) {
    if (j < ha.n_dense) {
      grp = lx_add(grp, lx_mul(ha.htab[(codes >> (2 * j)) & 3ull], xd[j]));
      if (++in == 4 || j == ha.n_dense - 1) {
        D = lx_add(D, grp);
        grp = 0.0f;
        in = 0;
      }
    }
  }
  return D;
}

// The head over a tile: the block's rows (a slice) for its 32 tokens; each warp takes rows
// w, w + XW, ... and keeps each lane's (token's) first maximum; the warps' maxima are combined in
// row order (the slice's maximum is the first among the warps' by value, then by row).
__global__ void __launch_bounds__(XW * 32) lpf_head_tile(PV pv, HeadArgs ha, Buf b) {
  extern __shared__ __align__(16) uint16_t xs[];
  __shared__ float s_best[XW][XT];
  __shared__ int s_bi[XW][XT];
  const int t0 = blockIdx.x * XT;
  fill_tile(xs, b.xn, b.Tp, t0);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ns = gridDim.y, k = blockIdx.y;
  const int r0 = (int)((long long)ha.V * k / ns), r1 = (int)((long long)ha.V * (k + 1) / ns);
  float xd[LXB_PF_MAXDENSE];
#pragma unroll
  for (int j = 0; j < LXB_PF_MAXDENSE; j++)
    xd[j] = j < ha.n_dense ? bf(xs[ha.dense_cols[j] * XT + lane]) : 0.0f;
  const int32_t* hp = pv.i32 + ha.head_ptr;
  float best = 0.0f;
  int bi = -1;
  for (int row = r0 + warp; row < r1; row += XW) {
    const int e0 = __ldg(hp + row), e1 = __ldg(hp + row + 1);
    float D = 0.0f;
    if (ha.n_dense) D = head_dense(ha, __ldg(pv.hcodes + row), xd);
    const float S = tdot(pv.ent + e0, (uint32_t)(e1 - e0), xs, lane);
    const float lg = lx_rbf(lx_add(D, S));
    if (bi < 0 || lg > best) {
      best = lg;
      bi = row;
    }
  }
  s_best[warp][lane] = best;
  s_bi[warp][lane] = bi;
  __syncthreads();
  if (warp == 0) {
    float v = 0.0f;
    int vi = -1;
    for (int w = 0; w < XW; w++) {  // equal logits: the lowest row wins (the first maximum)
      const int wi = s_bi[w][lane];
      const float wv = s_best[w][lane];
      if (wi >= 0 && (vi < 0 || wv > v || (wv == v && wi < vi))) {
        v = wv;
        vi = wi;
      }
    }
    b.hp[(size_t)k * b.Tp + t0 + lane] = make_uint2(__float_as_uint(v), (uint32_t)vi);
  }
}

// the slices' maxima in row order -> the prediction; with tokens, the first position whose
// prediction is not the next token
__global__ void __launch_bounds__(128) lpf_head_reduce(int ns, Buf b, int32_t* __restrict__ preds,
                                                       const int32_t* __restrict__ tok) {
  const int t = blockIdx.x * 128 + threadIdx.x;
  if (t >= b.T) return;
  float best = 0.0f;
  int bi = -1;
  for (int k = 0; k < ns; k++) {
    const uint2 p = b.hp[(size_t)k * b.Tp + t];
    if ((int)p.y < 0) continue;
    const float v = __uint_as_float(p.x);
    if (bi < 0 || v > best) {
      best = v;
      bi = (int)p.y;
    }
  }
  preds[t] = bi;
  if (tok && b.t_off + t + 1 < b.T_call && bi != tok[t + 1]) atomicMin(b.fw, b.t_off + t);
}

__global__ void lpf_fw_init(int* fw) { *fw = INT_MAX; }
__global__ void lpf_fw_done(const int* fw, int32_t* out) { *out = *fw == INT_MAX ? -1 : *fw; }

}  // namespace

// =============================================================================================
// The C ABI
// =============================================================================================
struct lxb_prefill_plan {
  int device;
  void* dimage;
  size_t bytes;
  lxb_pf_header hdr;
  PV pv;
  const lxb_pf_layer* dlayers;   // device
  lxb_pf_layer* hlayers;         // host copy
  uint32_t* status;
  cudaStream_t side;             // the decay scans run here, beside the layer stages
  cudaEvent_t* ev;               // per layer: gates done, state done (the recurrence's rows and
  int n_ev;                      // the conv windows, for the next view)
  static const int NSUB = 4;     // a long chunk runs as this many views, one stream each
  cudaStream_t sub[NSUB];
  cudaEvent_t evx[2 + NSUB];     // fork, the scans' end, the views' ends
  // per-stage timing (lxb_prefill_set_timing): an event pair around every launch
  int timing;
  static const int TCAP = 1024;
  cudaEvent_t tev[2 * TCAP];
  int tstage[TCAP];
  int n_t, n_tev;
  double tms[LXB_PF_STAGES];
  long long tcount[LXB_PF_STAGES];
};

namespace {

int cuda_rc(cudaError_t e) { return e == cudaSuccess ? LXB_OK : (int)e; }

// --- image validation: every offset, count and index the kernels follow ----------------------
struct PView {
  const unsigned char* base;
  size_t bytes;
  const lxb_pf_header* h;
  template <class T>
  const T* sec(int k) const { return reinterpret_cast<const T*>(base + h->sec[k].off); }
  int64_t n(int k) const { return h->sec[k].count; }
};

bool ent_ok(const PView& v, int64_t off, int64_t cnt) {
  return off >= 0 && cnt >= 0 && off + cnt <= v.n(LXB_PF_SEC_ENT);
}
bool i32_ok(const PView& v, int64_t off, int64_t cnt) {
  return off >= 0 && cnt >= 0 && off + cnt <= v.n(LXB_PF_SEC_I32);
}
bool u16_ok(const PView& v, int64_t off, int64_t cnt) {
  return off >= 0 && cnt >= 0 && off + cnt <= v.n(LXB_PF_SEC_U16);
}
// entries [off, off + cnt) exist and each index is below lim
bool ents_below(const PView& v, int64_t off, int64_t cnt, uint32_t lim) {
  if (!ent_ok(v, off, cnt)) return false;
  const uint32_t* e = v.sec<uint32_t>(LXB_PF_SEC_ENT) + off;
  for (int64_t k = 0; k < cnt; k++)
    if ((e[k] & 0xffffu) >= lim) return false;
  return true;
}
// n + 1 nondecreasing entry pointers at i32 offset p, the entries' indices below lim
bool ptrs_ok(const PView& v, int64_t p, int64_t n, uint32_t lim) {
  if (!i32_ok(v, p, n + 1)) return false;
  const int32_t* q = v.sec<int32_t>(LXB_PF_SEC_I32) + p;
  for (int64_t k = 0; k < n; k++)
    if (q[k + 1] < q[k]) return false;
  return ents_below(v, q[0], (int64_t)q[n] - q[0], lim);
}

bool validate(const unsigned char* img, size_t bytes) {
  if (!img || bytes < sizeof(lxb_pf_header) || (reinterpret_cast<uintptr_t>(img) & 7)) return false;
  PView v{img, bytes, reinterpret_cast<const lxb_pf_header*>(img)};
  const lxb_pf_header& h = *v.h;
  if (h.magic != LXB_PF_MAGIC || h.version != LXB_PF_VERSION || h.hidden != H) return false;
  if (h.n_layers < 1 || h.n_layers > 4096 || h.n_vocab < 1 || h.n_dense < 0 ||
      h.n_dense > LXB_PF_MAXDENSE || h.offset < 0 || h.n_embed_rows < (int64_t)h.offset + 1)
    return false;
  if (h.max_tap < 0 || h.max_lvh < 0 || h.max_lvh > NK * R || h.max_slot < 0 ||
      h.max_units < 0 || h.max_units > 65536)
    return false;
  const size_t esz[LXB_PF_SEC_COUNT] = {sizeof(lxb_pf_layer), 4, 4, 2, sizeof(lxb_pf_tap),
                                        sizeof(lxb_pf_vh), sizeof(lxb_pf_unit), 8};
  for (int k = 0; k < LXB_PF_SEC_COUNT; k++) {
    const lxb_pf_sec s = h.sec[k];
    if (s.off < (int64_t)sizeof(lxb_pf_header) || (s.off & 15) || s.count < 0 ||
        (uint64_t)s.count > (bytes / esz[k]) || (uint64_t)s.off + (uint64_t)s.count * esz[k] > bytes)
      return false;
  }
  if (v.n(LXB_PF_SEC_LAYERS) != h.n_layers || v.n(LXB_PF_SEC_VHS) != (int64_t)h.n_layers * NV)
    return false;
  if (!u16_ok(v, h.final_norm, H) || !ptrs_ok(v, h.head_ptr, h.n_vocab, H)) return false;
  if (h.n_dense) {
    if (v.n(LXB_PF_SEC_HCODES) != h.n_vocab) return false;
    for (int j = 0; j < h.n_dense; j++)
      if (h.dense_cols[j] < 0 || h.dense_cols[j] >= H) return false;
  }
  const lxb_pf_layer* lys = v.sec<lxb_pf_layer>(LXB_PF_SEC_LAYERS);
  const lxb_pf_tap* taps = v.sec<lxb_pf_tap>(LXB_PF_SEC_TAPS);
  const lxb_pf_vh* vhs = v.sec<lxb_pf_vh>(LXB_PF_SEC_VHS);
  const lxb_pf_unit* units = v.sec<lxb_pf_unit>(LXB_PF_SEC_UNITS);
  const int32_t* i32 = v.sec<int32_t>(LXB_PF_SEC_I32);
  for (int L = 0; L < h.n_layers; L++) {
    const lxb_pf_layer& ly = lys[L];
    if (!u16_ok(v, ly.ln_in, H) || !u16_ok(v, ly.ln_post, H) || !u16_ok(v, ly.gnorm, VD))
      return false;
    if (ly.n_tap < 0 || ly.n_tap > h.max_tap || ly.tap0 < 0 ||
        (int64_t)ly.tap0 + ly.n_tap > v.n(LXB_PF_SEC_TAPS))
      return false;
    for (int k = 0; k < ly.n_tap; k++) {
      const lxb_pf_tap& tp = taps[ly.tap0 + k];
      if (tp.conv_ch >= (uint32_t)CONV || !ents_below(v, tp.ent, tp.n, H)) return false;
    }
    if (!i32_ok(v, ly.chan, 3 * (int64_t)CONV)) return false;
    for (int c = 0; c < CONV; c++) {
      const int32_t* cc = i32 + ly.chan + 3 * c;
      if (cc[0] < -1 || cc[0] >= ly.n_tap || !ents_below(v, cc[1], cc[2], H)) return false;
    }
    if (ly.n_kh < 0 || ly.n_kh > NK || ly.n_slot < 0 || ly.n_slot > h.max_slot ||
        ly.n_kh * R > h.max_lvh || ly.nl < 0 || ly.nl > LXB_PF_MAXLIVE)
      return false;
    if (!i32_ok(v, ly.khs, 3 * (int64_t)ly.n_kh) || !i32_ok(v, ly.slots, 3 * (int64_t)ly.n_slot) ||
        !i32_ok(v, ly.livemask, NK * 8))
      return false;
    for (int k = 0; k < ly.n_kh; k++) {
      const int32_t* kh = i32 + ly.khs + 3 * k;
      if (kh[0] < 0 || kh[0] >= NK || kh[2] < 1 || kh[2] > ly.nl || kh[1] < 0 ||
          (int64_t)kh[1] + kh[2] > ly.n_slot)
        return false;
    }
    for (int k = 0; k < ly.n_slot; k++) {
      const int32_t* s = i32 + ly.slots + 3 * k;
      if (s[0] < 0 || s[0] >= KD || s[1] < -1 || s[1] >= ly.n_tap || s[2] < -1 ||
          s[2] >= ly.n_tap)
        return false;
    }
    const int64_t nd = (int64_t)ly.n_kh * R * VD;  // live value dims
    if (!i32_ok(v, ly.vtap, nd) || !i32_ok(v, ly.zrow, 2 * nd)) return false;
    for (int64_t k = 0; k < nd; k++) {
      const int32_t vt = i32[ly.vtap + k];
      if (vt < -1 || vt >= ly.n_tap) return false;
      if (!ents_below(v, i32[ly.zrow + 2 * k], i32[ly.zrow + 2 * k + 1], H)) return false;
    }
    if (!ptrs_ok(v, ly.out_ptr, H, (uint32_t)nd)) return false;
    for (int k = 0; k < NV; k++) {
      const lxb_pf_vh& p = vhs[(size_t)L * NV + k];
      if (!ents_below(v, p.a_ent, p.a_n, H) || !ents_below(v, p.b_ent, p.b_n, H)) return false;
    }
    if (ly.n_units < 0 || ly.n_units > h.max_units || ly.unit0 < 0 ||
        (int64_t)ly.unit0 + ly.n_units > v.n(LXB_PF_SEC_UNITS))
      return false;
    for (int k = 0; k < ly.n_units; k++) {
      const lxb_pf_unit& u = units[ly.unit0 + k];
      if ((uint64_t)u.u != (uint64_t)u.g + u.ng || !ents_below(v, u.g, (int64_t)u.ng + u.nu, H))
        return false;
    }
    if (!ptrs_ok(v, ly.down_ptr, H, (uint32_t)ly.n_units)) return false;
  }
  return true;
}

// scratch layout for a chunk of T tokens (byte offsets, each 256-aligned)
struct Layout {
  int Tp, ns;
  size_t x, xn, P, Y, e, beta, qs, ks, qm, km, o, on, hb, hp, flags, fw, total;
};

Layout layout(const lxb_pf_header& h, int T) {
  Layout l{};
  l.Tp = (T + TPAD - 1) / TPAD * TPAD;
  l.ns = std::min(512, std::max(1, (h.n_vocab + HEAD_ROWS - 1) / HEAD_ROWS));
  const size_t Tp = (size_t)l.Tp;
  size_t pos = 0;
  auto take = [&](size_t bytes) {
    const size_t at = pos;
    pos += (bytes + 255) & ~(size_t)255;
    return at;
  };
  l.x = take(2 * H * Tp);
  l.xn = take(2 * H * Tp);
  l.P = take(2 * (size_t)h.max_tap * Tp);
  l.Y = take(2 * (size_t)h.max_tap * Tp);
  l.e = take(4 * (size_t)h.n_layers * NV * Tp);
  l.beta = take(4 * (size_t)NV * Tp);
  l.qs = take(4 * (size_t)h.max_slot * Tp);
  l.ks = take(4 * (size_t)h.max_slot * Tp);
  l.qm = take(4 * (size_t)NK * Tp);
  l.km = take(4 * (size_t)NK * Tp);
  l.o = take(2 * (size_t)h.max_lvh * VD * Tp);
  l.on = take(2 * (size_t)h.max_lvh * VD * Tp);
  l.hb = take(2 * (size_t)h.max_units * Tp);
  l.hp = take(8 * (size_t)l.ns * Tp);
  l.flags = take(4 * (size_t)lxb_prefill_plan::NSUB * h.n_layers * NV);
  l.fw = take(16);
  l.total = pos;
  return l;
}

Buf buffers(const Layout& l, void* scratch, int T) {
  unsigned char* s = static_cast<unsigned char*>(scratch);
  Buf b;
  b.T = T;
  b.Tp = l.Tp;
  b.Te = l.Tp;
  b.t_off = 0;
  b.T_call = T;
  b.x = reinterpret_cast<uint16_t*>(s + l.x);
  b.xn = reinterpret_cast<uint16_t*>(s + l.xn);
  b.P = reinterpret_cast<uint16_t*>(s + l.P);
  b.Y = reinterpret_cast<uint16_t*>(s + l.Y);
  b.e = reinterpret_cast<float*>(s + l.e);
  b.beta = reinterpret_cast<float*>(s + l.beta);
  b.qs = reinterpret_cast<float*>(s + l.qs);
  b.ks = reinterpret_cast<float*>(s + l.ks);
  b.qm = reinterpret_cast<uint32_t*>(s + l.qm);
  b.km = reinterpret_cast<uint32_t*>(s + l.km);
  b.o = reinterpret_cast<uint16_t*>(s + l.o);
  b.on = reinterpret_cast<uint16_t*>(s + l.on);
  b.hb = reinterpret_cast<uint16_t*>(s + l.hb);
  b.hp = reinterpret_cast<uint2*>(s + l.hp);
  b.flags = reinterpret_cast<uint32_t*>(s + l.flags);
  b.fw = reinterpret_cast<int*>(s + l.fw);
  b.os = 0;  // set by the caller (the plan's max_lvh x 128)
  return b;
}

// The view of tokens [off, off + T) of a whole call's buffers (off a multiple of 256): the same
// strides, every per-token pointer moved by off, its own flags (view k of NSUB).
Buf view(const Buf& w, int off, int T, int k, int n_layers) {
  Buf b = w;
  b.T = T;
  b.Te = (T + TPAD - 1) / TPAD * TPAD;
  b.t_off = off;
  b.x += off;
  b.xn += off;
  b.P += off;
  b.Y += off;
  b.e += off;
  b.beta += off;
  b.qs += off;
  b.ks += off;
  b.qm += off;
  b.km += off;
  b.o += (size_t)off * w.os;
  b.on += off;
  b.hb += off;
  b.hp += off;
  b.flags += (size_t)k * n_layers * NV;
  return b;
}

#define LPF_TRY(x)                      \
  do {                                  \
    cudaError_t e_ = (x);               \
    if (e_ != cudaSuccess) return cuda_rc(e_); \
  } while (0)
#define LPF_LAUNCHED() LPF_TRY(cudaGetLastError())

int timing_begin(lxb_prefill_plan* p, cudaStream_t s) {
  if (!p->timing || p->n_t >= lxb_prefill_plan::TCAP || 2 * p->n_t + 1 >= p->n_tev) return -1;
  if (cudaEventRecord(p->tev[2 * p->n_t], s)) return -1;
  return p->n_t;
}
void timing_end(lxb_prefill_plan* p, int i, int stage, cudaStream_t s) {
  if (i < 0) return;
  if (cudaEventRecord(p->tev[2 * i + 1], s)) return;
  p->tstage[i] = stage;
  p->n_t = i + 1;
}
// one stage launch: the launch, its error check and, with timing on, an event pair around it
#define LPF_STAGE(k, s, launch)            \
  do {                                     \
    const int ti_ = timing_begin(p, s);    \
    launch;                                \
    LPF_LAUNCHED();                        \
    timing_end(p, ti_, k, s);              \
  } while (0)

// Layer L's stages over one view b on stream st: the decay scan forks to the plan's second stream
// after the gates; with chained views, the state's part (conv windows, recurrence) waits for the
// previous view's (wait_prev: ev[2L + 1]) and then marks its own done (mark_done).
int layer_stages(lxb_prefill_plan* p, const uint64_t* sp, const Buf& b, cudaStream_t st, int L,
                 bool wait_prev, bool mark_done) {
  const lxb_pf_header& h = p->hdr;
  const int nb128 = (b.T + 127) / 128, nbrow = b.Te / ROWT;
  const lxb_pf_layer& ly = p->hlayers[L];
  const lxb_pf_layer* dly = p->dlayers + L;
  LPF_STAGE(LXB_PF_NORM, st, (lpf_norm<<<(b.T + 31) / 32, 512, 0, st>>>(b.x, b.T, b.Tp, p->pv.u16 + ly.ln_in, h.eps, b.xn)));
  if (ly.n_tap) {
    LPF_STAGE(LXB_PF_TAPS, st, (lpf_taps<<<dim3(nbrow, ly.n_tap), 128, 0, st>>>(p->pv, ly.tap0, b)));
  }
  LPF_STAGE(LXB_PF_GATES, st, (lpf_gates<<<dim3(nbrow, NV), 128, 0, st>>>(p->pv, L, b)));
  // the decay of the other rows, on the side stream from here on (in view order per layer)
  LPF_TRY(cudaEventRecord(p->ev[2 * L], st));
  LPF_TRY(cudaStreamWaitEvent(p->side, p->ev[2 * L], 0));
  LPF_STAGE(LXB_PF_SCAN, p->side, (lpf_scan<<<dim3(NV, KD / 8), 256, 0, p->side>>>(p->pv, dly, L, sp, b)));
  if (wait_prev) LPF_TRY(cudaStreamWaitEvent(st, p->ev[2 * L + 1], 0));
  if (ly.n_tap) {
    LPF_STAGE(LXB_PF_CONV, st, (lpf_conv<<<dim3(nbrow, ly.n_tap), 128, 0, st>>>(p->pv, ly.tap0, sp, L, b)));
  }
  LPF_STAGE(LXB_PF_WINDOWS, st, (lpf_windows<<<CONV / 128, 128, 0, st>>>(p->pv, dly, sp, L, b)));
  if (ly.n_kh) {
    LPF_STAGE(LXB_PF_QK, st, (lpf_qk<<<dim3(nb128, ly.n_kh), 128, 0, st>>>(p->pv, dly, b)));
    const int g = ly.n_kh * R;
    switch (ly.nl) {  // the register slots: the layer's most live rows, rounded up a little
#define LPF_R(n) LPF_STAGE(LXB_PF_RECUR, st, (lpf_recur<n><<<g, 128, 0, st>>>(p->pv, dly, L, sp, b))); break
      case 1: case 2: LPF_R(2);
      case 3: LPF_R(3);
      case 4: LPF_R(4);
      case 5: LPF_R(5);
      case 6: LPF_R(6);
      case 7: case 8: LPF_R(8);
      case 9: case 10: case 11: case 12: LPF_R(12);
      case 13: case 14: case 15: case 16: LPF_R(16);
      case 17: case 18: case 19: case 20: case 21: case 22: case 23: case 24: LPF_R(24);
      default: LPF_R(31);
#undef LPF_R
    }
  }
  if (mark_done) LPF_TRY(cudaEventRecord(p->ev[2 * L + 1], st));
  if (ly.n_kh) {
    const int g = ly.n_kh * R;
    LPF_STAGE(LXB_PF_GNORM, st, (lpf_gnorm<<<dim3(g, nbrow), 128, 0, st>>>(p->pv, dly, h.eps, b)));
    LPF_STAGE(LXB_PF_OUT, st, (lpf_add_rows<<<dim3(H, nbrow), 128, 0, st>>>(p->pv, ly.out_ptr, b.on, b)));
  }
  if (ly.n_units) {
    LPF_STAGE(LXB_PF_NORM, st, (lpf_norm<<<(b.T + 31) / 32, 512, 0, st>>>(b.x, b.T, b.Tp, p->pv.u16 + ly.ln_post, h.eps, b.xn)));
    LPF_STAGE(LXB_PF_MLP, st, (lpf_mlp_tile<<<b.Te / XT, XW * 32, XSMEM, st>>>(p->pv, ly.unit0, ly.n_units, b)));
    LPF_STAGE(LXB_PF_DOWN, st, (lpf_add_rows<<<dim3(H, nbrow), 128, 0, st>>>(p->pv, ly.down_ptr, b.hb, b)));
  }
  return LXB_OK;
}

int run_head(lxb_prefill_plan* p, const Buf& b, const Layout& l, int32_t* preds,
             const int32_t* tok, cudaStream_t st);

// The views of a chunk: a chunk of at least 4 x 2,048 tokens runs as NSUB views of equal size
// (multiples of 256), view k on the plan's stream k. Per layer the views' state parts are chained
// (view k's conv windows and recurrence wait for view k - 1's), everything else of a view is
// its own, so layer L + 1 of view k runs beside layer L of view k + 1: the recurrences (a
// dependent chain per token on few warps) overlap the token-parallel stages of other views.
int n_views(int T) { return T >= lxb_prefill_plan::NSUB * 2048 ? lxb_prefill_plan::NSUB : 1; }

// The chip layers over the call's rows in w.x (feature-major), updating the state in place;
// with preds, also the head (tok: the call's token ids for the mismatch check, or NULL). Every
// stream of the plan is joined back into st before it returns.
int run_chunk(lxb_prefill_plan* p, const uint64_t* sp, const Buf& w, const Layout& l,
              cudaStream_t st, int32_t* preds, const int32_t* tok) {
  const lxb_pf_header& h = p->hdr;
  const int nv = n_views(w.T);
  LPF_TRY(cudaMemsetAsync(w.flags, 0, 4 * (size_t)nv * h.n_layers * NV, st));
  if (nv == 1) {
    for (int L = 0; L < h.n_layers; L++) {
      int rc = layer_stages(p, sp, w, st, L, false, false);
      if (rc) return rc;
    }
    if (preds) {
      int rc = run_head(p, w, l, preds, tok, st);
      if (rc) return rc;
    }
  } else {
    const int per = (w.T / nv + TPAD - 1) / TPAD * TPAD;
    LPF_TRY(cudaEventRecord(p->evx[0], st));
    for (int k = 0; k < nv; k++) {
      const int off = k * per, n = std::min(per, w.T - off);
      if (n <= 0) break;
      cudaStream_t sk = p->sub[k];
      LPF_TRY(cudaStreamWaitEvent(sk, p->evx[0], 0));
      const Buf b = view(w, off, n, k, h.n_layers);
      for (int L = 0; L < h.n_layers; L++) {
        int rc = layer_stages(p, sp, b, sk, L, k > 0, true);
        if (rc) return rc;
      }
      if (preds) {
        int rc = run_head(p, b, l, preds + off, tok ? tok + off : nullptr, sk);
        if (rc) return rc;
      }
      LPF_TRY(cudaEventRecord(p->evx[2 + k], sk));
      LPF_TRY(cudaStreamWaitEvent(st, p->evx[2 + k], 0));
    }
  }
  LPF_TRY(cudaEventRecord(p->evx[1], p->side));
  LPF_TRY(cudaStreamWaitEvent(st, p->evx[1], 0));
  return LXB_OK;
}

int run_head(lxb_prefill_plan* p, const Buf& b, const Layout& l, int32_t* preds,
             const int32_t* tok, cudaStream_t st) {
  const lxb_pf_header& h = p->hdr;
  const int nb128 = (b.T + 127) / 128;
  LPF_STAGE(LXB_PF_NORM, st, (lpf_norm<<<(b.T + 31) / 32, 512, 0, st>>>(b.x, b.T, b.Tp, p->pv.u16 + h.final_norm, h.eps, b.xn)));
  HeadArgs ha;
  ha.V = h.n_vocab;
  ha.n_dense = h.n_dense;
  ha.head_ptr = h.head_ptr;
  memcpy(ha.htab, h.htab, sizeof(ha.htab));
  memcpy(ha.dense_cols, h.dense_cols, sizeof(ha.dense_cols));
  LPF_STAGE(LXB_PF_HEAD, st, (lpf_head_tile<<<dim3(b.Te / XT, l.ns), XW * 32, XSMEM, st>>>(p->pv, ha, b)));
  LPF_STAGE(LXB_PF_REDUCE, st, (lpf_head_reduce<<<nb128, 128, 0, st>>>(l.ns, b, preds, tok)));
  return LXB_OK;
}

}  // namespace

extern "C" int lxb_prefill_check_image(const void* image, size_t bytes) {
  return validate(static_cast<const unsigned char*>(image), bytes) ? LXB_OK : LXB_E_IMAGE;
}

extern "C" int lxb_prefill_plan_create(const void* image, size_t bytes, lxb_prefill_plan** out) {
  if (!out) return LXB_E_INVAL;
  *out = nullptr;
  const unsigned char* img = static_cast<const unsigned char*>(image);
  if (!validate(img, bytes)) return LXB_E_IMAGE;
  int dev = 0;
  LPF_TRY(cudaGetDevice(&dev));
  int major = 0;
  LPF_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  if (major < 10) return LXB_E_DEVICE;
  lxb_prefill_plan* p = new (std::nothrow) lxb_prefill_plan();
  if (!p) return LXB_E_INVAL;
  p->device = dev;
  p->bytes = bytes;
  memcpy(&p->hdr, img, sizeof(p->hdr));
  const lxb_pf_header& h = p->hdr;
  p->hlayers = new (std::nothrow) lxb_pf_layer[h.n_layers];
  p->n_ev = 2 * h.n_layers;
  p->ev = new (std::nothrow) cudaEvent_t[p->n_ev]();
  auto fail = [&](cudaError_t e) {
    lxb_prefill_plan_destroy(p);
    return e ? cuda_rc(e) : LXB_E_INVAL;
  };
  if (!p->hlayers || !p->ev) return fail(cudaSuccess);
  memcpy(p->hlayers, img + h.sec[LXB_PF_SEC_LAYERS].off, sizeof(lxb_pf_layer) * h.n_layers);
  cudaError_t e;
  if ((e = cudaMalloc(&p->dimage, bytes))) return fail(e);
  if ((e = cudaMemcpy(p->dimage, img, bytes, cudaMemcpyHostToDevice))) return fail(e);
  if ((e = cudaMalloc(&p->status, 16))) return fail(e);
  if ((e = cudaMemset(p->status, 0, 16))) return fail(e);
  if ((e = cudaFuncSetAttribute(lpf_mlp_tile, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                XSMEM)))
    return fail(e);
  if ((e = cudaFuncSetAttribute(lpf_head_tile, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                XSMEM)))
    return fail(e);
  int lo = 0, hi = 0;
  cudaDeviceGetStreamPriorityRange(&lo, &hi);
  if ((e = cudaStreamCreateWithPriority(&p->side, cudaStreamNonBlocking, lo))) return fail(e);
  for (int k = 0; k < p->n_ev; k++)
    if ((e = cudaEventCreateWithFlags(&p->ev[k], cudaEventDisableTiming))) return fail(e);
  for (int k = 0; k < lxb_prefill_plan::NSUB; k++)
    if ((e = cudaStreamCreateWithFlags(&p->sub[k], cudaStreamNonBlocking))) return fail(e);
  for (int k = 0; k < 2 + lxb_prefill_plan::NSUB; k++)
    if ((e = cudaEventCreateWithFlags(&p->evx[k], cudaEventDisableTiming))) return fail(e);
  const unsigned char* d = static_cast<const unsigned char*>(p->dimage);
  p->pv.layers = reinterpret_cast<const lxb_pf_layer*>(d + h.sec[LXB_PF_SEC_LAYERS].off);
  p->pv.ent = reinterpret_cast<const uint32_t*>(d + h.sec[LXB_PF_SEC_ENT].off);
  p->pv.i32 = reinterpret_cast<const int32_t*>(d + h.sec[LXB_PF_SEC_I32].off);
  p->pv.u16 = reinterpret_cast<const uint16_t*>(d + h.sec[LXB_PF_SEC_U16].off);
  p->pv.taps = reinterpret_cast<const lxb_pf_tap*>(d + h.sec[LXB_PF_SEC_TAPS].off);
  p->pv.vhs = reinterpret_cast<const lxb_pf_vh*>(d + h.sec[LXB_PF_SEC_VHS].off);
  p->pv.units = reinterpret_cast<const lxb_pf_unit*>(d + h.sec[LXB_PF_SEC_UNITS].off);
  p->pv.hcodes = reinterpret_cast<const unsigned long long*>(d + h.sec[LXB_PF_SEC_HCODES].off);
  p->pv.status = p->status;
  p->dlayers = p->pv.layers;
  *out = p;
  return LXB_OK;
}

extern "C" size_t lxb_prefill_scratch_bytes(const lxb_prefill_plan* p, int T) {
  if (!p || T < 1) return 0;
  return layout(p->hdr, T).total;
}

static int check_call(lxb_prefill_plan* p, void* scratch, int T) {
  if (!p || !scratch || T < 1 || T > LXB_PF_MAX_T) return LXB_E_INVAL;
  if (reinterpret_cast<uintptr_t>(scratch) & 255) return LXB_E_INVAL;
  int dev = -1;
  LPF_TRY(cudaGetDevice(&dev));
  return dev == p->device ? LXB_OK : LXB_E_INVAL;
}

extern "C" int lxb_prefill(lxb_prefill_plan* p, const uint64_t* state_ptrs, const uint16_t* embed,
                           const int32_t* tokens, int T, int32_t* preds, int32_t* first_wrong,
                           void* scratch, void* cuda_stream) {
  int rc = check_call(p, scratch, T);
  if (rc) return rc;
  if (!state_ptrs || !embed || !tokens || !preds) return LXB_E_INVAL;
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  const Layout l = layout(p->hdr, T);
  Buf b = buffers(l, scratch, T);
  b.os = p->hdr.max_lvh * VD;
  LPF_STAGE(LXB_PF_ROWS, st,
            (lpf_rows_in<<<dim3(l.Tp / 32, H / 32), 256, 0, st>>>(
                embed, tokens, p->hdr.offset, p->hdr.n_embed_rows, T, l.Tp, b.x, p->status)));
  if (first_wrong) {
    lpf_fw_init<<<1, 1, 0, st>>>(b.fw);
    LPF_LAUNCHED();
  }
  if ((rc = run_chunk(p, state_ptrs, b, l, st, preds, first_wrong ? tokens : nullptr))) return rc;
  if (first_wrong) {
    lpf_fw_done<<<1, 1, 0, st>>>(b.fw, first_wrong);
    LPF_LAUNCHED();
  }
  return LXB_OK;
}

extern "C" int lxb_prefill_layers(lxb_prefill_plan* p, const uint64_t* state_ptrs,
                                  const uint16_t* h_in, uint16_t* h_out, int T, void* scratch,
                                  void* cuda_stream) {
  int rc = check_call(p, scratch, T);
  if (rc) return rc;
  if (!state_ptrs || !h_in) return LXB_E_INVAL;
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  const Layout l = layout(p->hdr, T);
  Buf b = buffers(l, scratch, T);
  b.os = p->hdr.max_lvh * VD;
  LPF_STAGE(LXB_PF_ROWS, st,
            (lpf_rows_in<<<dim3(l.Tp / 32, H / 32), 256, 0, st>>>(h_in, nullptr, 0, T, T, l.Tp,
                                                                  b.x, p->status)));
  if ((rc = run_chunk(p, state_ptrs, b, l, st, nullptr, nullptr))) return rc;
  if (h_out) {
    LPF_STAGE(LXB_PF_ROWS, st,
              (lpf_rows_out<<<dim3(l.Tp / 32, H / 32), 256, 0, st>>>(b.x, T, l.Tp, h_out)));
  }
  return LXB_OK;
}

extern "C" int lxb_prefill_head(lxb_prefill_plan* p, const uint16_t* h, int T, int32_t* preds,
                                void* scratch, void* cuda_stream) {
  int rc = check_call(p, scratch, T);
  if (rc) return rc;
  if (!h || !preds) return LXB_E_INVAL;
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  const Layout l = layout(p->hdr, T);
  Buf b = buffers(l, scratch, T);
  b.os = p->hdr.max_lvh * VD;
  LPF_STAGE(LXB_PF_ROWS, st,
            (lpf_rows_in<<<dim3(l.Tp / 32, H / 32), 256, 0, st>>>(h, nullptr, 0, T, T, l.Tp,
                                                                  b.x, p->status)));
  return run_head(p, b, l, preds, nullptr, st);
}

extern "C" int lxb_prefill_status(lxb_prefill_plan* p, lxb_error* err) {
  if (!p || !err) return LXB_E_INVAL;
  uint32_t s[3];
  LPF_TRY(cudaMemcpy(s, p->status, 12, cudaMemcpyDeviceToHost));
  err->status = s[0];
  err->first_stream = (int32_t)s[1];
  err->first_step = (int32_t)s[2];
  return LXB_OK;
}

extern "C" int lxb_prefill_status_clear(lxb_prefill_plan* p) {
  if (!p) return LXB_E_INVAL;
  return cuda_rc(cudaMemset(p->status, 0, 16));
}

extern "C" int lxb_prefill_set_timing(lxb_prefill_plan* p, int on) {
  if (!p) return LXB_E_INVAL;
  if (on && !p->n_tev) {
    for (int k = 0; k < 2 * lxb_prefill_plan::TCAP; k++) {
      cudaError_t e = cudaEventCreate(&p->tev[k]);
      if (e) return cuda_rc(e);
      p->n_tev = k + 1;
    }
  }
  p->timing = on ? 1 : 0;
  return LXB_OK;
}

extern "C" int lxb_prefill_timing(lxb_prefill_plan* p, double* ms, long long* launches, int n) {
  if (!p || n < 0 || (n && (!ms || !launches))) return LXB_E_INVAL;
  for (int i = 0; i < p->n_t; i++) {
    float t = 0.0f;
    cudaError_t e = cudaEventSynchronize(p->tev[2 * i + 1]);
    if (!e) e = cudaEventElapsedTime(&t, p->tev[2 * i], p->tev[2 * i + 1]);
    if (e) return cuda_rc(e);
    p->tms[p->tstage[i]] += t;
    p->tcount[p->tstage[i]]++;
  }
  p->n_t = 0;
  for (int k = 0; k < n && k < LXB_PF_STAGES; k++) {
    ms[k] = p->tms[k];
    launches[k] = p->tcount[k];
    p->tms[k] = 0.0;
    p->tcount[k] = 0;
  }
  return LXB_OK;
}

extern "C" const char* lxb_prefill_stage_name(int k) {
  static const char* names[LXB_PF_STAGES] = {"rows", "norm", "taps", "gates", "scan", "conv",
                                             "windows", "qk", "recur", "gnorm", "out", "mlp",
                                             "down", "head", "reduce"};
  return k >= 0 && k < LXB_PF_STAGES ? names[k] : "";
}

extern "C" void lxb_prefill_plan_destroy(lxb_prefill_plan* p) {
  if (!p) return;
  for (int k = 0; k < p->n_tev; k++) cudaEventDestroy(p->tev[k]);
  if (p->ev)
    for (int k = 0; k < p->n_ev; k++)
      if (p->ev[k]) cudaEventDestroy(p->ev[k]);
  if (p->side) cudaStreamDestroy(p->side);
  for (int k = 0; k < lxb_prefill_plan::NSUB; k++)
    if (p->sub[k]) cudaStreamDestroy(p->sub[k]);
  for (int k = 0; k < 2 + lxb_prefill_plan::NSUB; k++)
    if (p->evx[k]) cudaEventDestroy(p->evx[k]);
  if (p->dimage) cudaFree(p->dimage);
  if (p->status) cudaFree(p->status);
  delete[] p->ev;
  delete[] p->hlayers;
  delete p;
}
