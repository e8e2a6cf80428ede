// TEST INFRASTRUCTURE ONLY: a CPU restatement of the chip decode step, used by tests/, by
// __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the checker. Nothing in the
// product path links or calls it.
//
// It restates the reference's stock decode (lx/lx/hf.py:169-184 driving transformers'
// Qwen3_5DecoderLayer; the GDN arithmetic is transformers' torch_causal_conv1d_update,
// l2norm and torch_recurrent_gated_delta_rule, modeling_qwen3_5.py:210-226, 228-231, 314-353,
// the gated norm 175-190, Qwen3_5RMSNorm 711-728), with the fp32 reductions in one fixed order
// that the CUDA kernels share, and the stock model's elementwise functions from lxb_math.h.
// Each rounding point is commented with the stock expression it follows. Per value head, the
// sums run over the nonzero terms only (adding +-0 to a partial sum that started at +0 leaves it
// unchanged), which is how the sparse kernels can skip the zeros and stay bit-identical.
//
// Reduction orders (the "canonical" orders; the kernels implement exactly these):
//   dot(row, x)    sequential over the row's entries in ascending column, from +0
//   SSQ (2560)     lane t of 512 sums x[t + 512 i]^2, i = 0..4 in order; xor butterfly over the
//                  32 lanes of each warp (16, 8, 4, 2, 1); xor butterfly over the 16 warp sums
//   l2 sum (256)   sequential over the nonzero squares in ascending index, from +0
//   gated-norm sum lane l of 32 sums o[4l..4l+3]^2 in order; xor butterfly over the lanes
//   kv, o          sequential over the rows with a nonzero key / query, ascending, from +0
//   head logit     D + S: D over the head's "dense" columns (nonzero in every row, at most 32,
//                  at most 4 distinct values) in groups of 4 ascending, each group sequential
//                  from +0 and the groups summed in order from +0; S over the row's other
//                  entries sequentially from +0. Without dense columns D = +0.
#include <stdbool.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "../linuxformer_b200/csrc/lxb_math.h"

#define H 2560
#define KD 256
#define VD 128
#define NK 16
#define NV 128
#define RR 8
#define CONV (2 * NK * KD + NV * VD)
#define ZD (NV * VD)

typedef struct {
  int64_t rows, cols;
  const int64_t* indptr;
  const int32_t* indices;
  const uint16_t* data;
} lxo_csr;

typedef struct {
  lxo_csr qkv, z, b, a, out, gate, up, down;
  const uint16_t* conv;  // [CONV][4]
  const uint16_t *A_log, *dt_bias, *gnorm, *ln_in, *ln_post;
} lxo_layer;

typedef struct {
  int n_layers;
  const lxo_layer* layers;
  const uint16_t* embed;
  int64_t n_embed;
  int offset;
  lxo_csr head;
  const uint16_t* final_norm;
  float eps;
} lxo_chip;

// sequential dot over a CSR row, from +0
static float row_dot(const lxo_csr* m, int64_t r, const float* x) {
  float s = 0.0f;
  for (int64_t e = m->indptr[r]; e < m->indptr[r + 1]; e++)
    s = lx_add(s, lx_mul(x[m->indices[e]], lx_f(m->data[e])));
  return s;
}

// the canonical 2560-element sum of squares
static float ssq2560(const float* x) {
  float lane[512];
  for (int t = 0; t < 512; t++) {
    float s = lx_mul(x[t], x[t]);
    for (int i = 1; i < 5; i++) s = lx_add(s, lx_mul(x[t + 512 * i], x[t + 512 * i]));
    lane[t] = s;
  }
  float w[16];
  for (int wp = 0; wp < 16; wp++) {
    float v[32];
    for (int l = 0; l < 32; l++) v[l] = lane[wp * 32 + l];
    for (int off = 16; off > 0; off >>= 1) {
      float nv[32];
      for (int l = 0; l < 32; l++) nv[l] = lx_add(v[l], v[l ^ off]);
      memcpy(v, nv, sizeof(v));
    }
    w[wp] = v[0];
  }
  for (int off = 8; off > 0; off >>= 1) {
    float nw[16];
    for (int l = 0; l < 16; l++) nw[l] = lx_add(w[l], w[l ^ off]);
    memcpy(w, nw, sizeof(w));
  }
  return w[0];
}

// Qwen3_5RMSNorm(x) -> bf16 values: x * rsqrt(mean(x^2) + eps) * (1 + w)   (modeling 711-728)
static void rms_norm(const float* x, const uint16_t* w, float eps, float* out) {
  const float ms = lx_div(ssq2560(x), (float)H);
  const float r = lx_rsqrt(lx_add(ms, eps));
  for (int c = 0; c < H; c++) {
    const float w1 = lx_add(1.0f, lx_f(w[c]));
    out[c] = lx_rbf(lx_mul(lx_mul(x[c], r), w1));
  }
}

// the gated norm's sum of 128 squares: lane l sums 4 in order, then an xor butterfly
static float sumsq128(const float* o) {
  float v[32];
  for (int l = 0; l < 32; l++) {
    float s = lx_mul(o[4 * l], o[4 * l]);
    for (int i = 1; i < 4; i++) s = lx_add(s, lx_mul(o[4 * l + i], o[4 * l + i]));
    v[l] = s;
  }
  for (int off = 16; off > 0; off >>= 1) {
    float nv[32];
    for (int l = 0; l < 32; l++) nv[l] = lx_add(v[l], v[l ^ off]);
    memcpy(v, nv, sizeof(v));
  }
  return v[0];
}

// transformers l2norm on a bf16 vector: x * rsqrt(sum(x * x) + 1e-6), every op in bf16
// (modeling 228-231; the query/key are bf16 there), then to fp32
static void l2norm_bf16(const float* x, int n, float* out) {
  float s = 0.0f;
  for (int i = 0; i < n; i++) {
    const float sq = lx_rbf(lx_mul(x[i], x[i]));
    if (sq != 0.0f) s = lx_add(s, sq);
  }
  const float sb = lx_rbf(s);
  const float se = lx_rbf(lx_add(sb, 1e-6f));
  const float inv = lx_rbf(lx_rsqrt(se));
  for (int i = 0; i < n; i++) out[i] = lx_rbf(lx_mul(x[i], inv));
}

typedef struct {
  const lxo_chip* chip;
  float* rec;     // [L][NV][KD][VD]
  uint16_t* conv; // [L][CONV][4]
  // scratch
  float x[H], xn[H];
  float qkv[CONV];
  float on[ZD];
  int dense_cols[32];
  int n_dense;
  int64_t* cnt;  // this step's counters (LXO_C_*), or NULL
  float* xin;    // this step's GDN input rows [n_layers][H], or NULL
  int32_t* act;  // this step's per-(layer, key head) activity bits, [n_layers][16], or NULL
} lxo_run;

// per-step activity counters: what the step logically reads and writes (the bench's algorithmic
// bytes per token are computed from them)
enum {
  LXO_C_CHANS,     // live conv channels (window read + write: 16 bytes each)
  LXO_C_QKV_ENT,   // in_proj_qkv entries of the live channels
  LXO_C_BA_ENT,    // in_proj_b / in_proj_a entries of the value heads evaluated
  LXO_C_Z_ENT,     // in_proj_z entries of the value heads with output
  LXO_C_ROWS,      // recurrent-state rows touched (decayed or keyed or queried; 512 B each)
  LXO_C_OUT_ENT,   // out_proj entries with a nonzero input
  LXO_C_GU_ENT,    // gate / up entries of the live units
  LXO_C_DOWN_ENT,  // down_proj entries with a nonzero input
  LXO_C_HEAD_B,    // head bytes (8 per row of dense codes, 4 per sparse entry)
  LXO_C_VH_ACTIVE, // value heads with a nonzero query or key
  LXO_C_VH_WRITE,  // value heads whose state took a key update
  LXO_C_VH_OUT,    // value heads with output
  LXO_C_GDN_WRITE, // layers whose GDN changed the residual
  LXO_C_N
};

// one GDN layer on the residual x (in place)
static void gdn_layer(lxo_run* st, int L) {
  const lxo_chip* chip = st->chip;
  const lxo_layer* ly = &chip->layers[L];
  float* x = st->x;
  float* xn = st->xn;
  if (st->xin) memcpy(st->xin + (size_t)L * H, x, sizeof(float) * H);
  rms_norm(x, ly->ln_in, chip->eps, xn);
  // in_proj_qkv, then torch_causal_conv1d_update: window [w0 w1 w2 w3] -> [w1 w2 w3 P],
  // out = silu(conv over the new window) in bf16
  uint16_t* cw = st->conv + (size_t)L * CONV * 4;
  int64_t n_ch = 0, n_ent = 0;
#pragma omp parallel for schedule(static) reduction(+ : n_ch, n_ent)
  for (int ch = 0; ch < CONV; ch++) {
    const bool live = ly->qkv.indptr[ch + 1] > ly->qkv.indptr[ch];
    if (!live) {  // a zero row: P = 0 every step; its window only ever holds what it held
      st->qkv[ch] = 0.0f;
      bool any = false;
      for (int j = 0; j < 4; j++) any |= (cw[ch * 4 + j] & 0x7fff) != 0;
      if (!any) continue;
    }
    const uint16_t P = lx_rb(row_dot(&ly->qkv, ch, xn));
    n_ch++;
    n_ent += ly->qkv.indptr[ch + 1] - ly->qkv.indptr[ch];
    uint16_t* w = cw + (size_t)ch * 4;
    const uint16_t n0 = w[1], n1 = w[2], n2 = w[3];
    w[0] = n0;
    w[1] = n1;
    w[2] = n2;
    w[3] = P;
    const uint16_t* k = ly->conv + (size_t)ch * 4;
    float y = 0.0f;
    y = lx_add(y, lx_mul(lx_f(k[0]), lx_f(n0)));
    y = lx_add(y, lx_mul(lx_f(k[1]), lx_f(n1)));
    y = lx_add(y, lx_mul(lx_f(k[2]), lx_f(n2)));
    y = lx_add(y, lx_mul(lx_f(k[3]), lx_f(P)));
    st->qkv[ch] = lx_rbf(lx_silu(lx_rbf(y)));
  }
  memset(st->on, 0, sizeof(st->on));
  int any_out = 0;
  int64_t c_ba = 0, c_z = 0, c_rows = 0, c_act = 0, c_wr = 0, c_out = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : any_out) \
    reduction(+ : c_ba, c_z, c_rows, c_act, c_wr, c_out)
  for (int kh = 0; kh < NK; kh++) {
    const float* q = st->qkv + kh * KD;
    const float* k = st->qkv + NK * KD + kh * KD;
    int qa = 0, ka = 0;
    for (int i = 0; i < KD; i++) {
      qa |= q[i] != 0.0f;
      ka |= k[i] != 0.0f;
    }
    float qn[KD], kn[KD];
    if (qa) l2norm_bf16(q, KD, qn);
    if (ka) l2norm_bf16(k, KD, kn);
    int anyg_h = 0, out_h = 0;
    for (int r = 0; r < RR; r++) {
      const int vh = kh * RR + r;
      // beta = sigmoid(in_proj_b(x)) in bf16; g = -exp(A_log) * softplus(a + dt_bias) in fp32
      const float bb = lx_rbf(row_dot(&ly->b, vh, xn));
      const float beta = lx_rbf(lx_sigmoid(bb));
      const float a = lx_rbf(row_dot(&ly->a, vh, xn));
      const float A = -lx_exp(lx_f(ly->A_log[vh]));
      const float g = lx_mul(A, lx_softplus(lx_add(a, lx_f(ly->dt_bias[vh]))));
      anyg_h |= g != 0.0f;
      c_ba += ly->a.indptr[vh + 1] - ly->a.indptr[vh];
      if (!qa && !ka && g == 0.0f) continue;  // the state stays, o = 0
      c_ba += ly->b.indptr[vh + 1] - ly->b.indptr[vh];
      c_act += qa || ka;
      c_wr += ka;
      float* S = st->rec + (((size_t)L * NV + vh) * KD) * VD;
      for (int i = 0; i < KD; i++) {  // rows touched: nonzero rows decayed, keyed or queried
        int nzr = 0;
        if (g != 0.0f)
          for (int j = 0; j < VD; j++) nzr |= S[i * VD + j] != 0.0f;
        c_rows += nzr || (ka && kn[i] != 0.0f) || (qa && qn[i] != 0.0f);
      }
      if (g != 0.0f) {
        const float e = lx_exp(g);
        for (int i = 0; i < KD * VD; i++) S[i] = lx_mul(S[i], e);
      }
      const float* v = st->qkv + 2 * NK * KD + vh * VD;
      float o[VD];
      for (int j = 0; j < VD; j++) {
        if (ka) {
          float kv = 0.0f;
          for (int i = 0; i < KD; i++)
            if (kn[i] != 0.0f) kv = lx_add(kv, lx_mul(S[i * VD + j], kn[i]));
          const float delta = lx_mul(lx_sub(v[j], kv), beta);
          for (int i = 0; i < KD; i++)
            if (kn[i] != 0.0f) S[i * VD + j] = lx_add(S[i * VD + j], lx_mul(kn[i], delta));
        }
        float oo = 0.0f;
        if (qa)
          for (int i = 0; i < KD; i++)
            if (qn[i] != 0.0f) oo = lx_add(oo, lx_mul(S[i * VD + j], lx_mul(qn[i], 0.0625f)));
        o[j] = lx_rbf(oo);
      }
      int nz = 0;
      for (int j = 0; j < VD; j++) nz |= o[j] != 0.0f;
      if (!nz) continue;
      // Qwen3_5RMSNormGated(o, z): bf16(bf16(w * bf16(o * rsqrt(mean(o^2) + eps))) * silu(z))
      const float var = lx_div(sumsq128(o), 128.0f);
      const float rr = lx_rsqrt(lx_add(var, chip->eps));
      for (int j = 0; j < VD; j++) {
        const float hn = lx_rbf(lx_mul(o[j], rr));
        const float u = lx_rbf(lx_mul(lx_f(ly->gnorm[j]), hn));
        const float z = lx_rbf(row_dot(&ly->z, (int64_t)vh * VD + j, xn));
        c_z += ly->z.indptr[(int64_t)vh * VD + j + 1] - ly->z.indptr[(int64_t)vh * VD + j];
        st->on[vh * VD + j] = lx_rbf(lx_mul(u, lx_silu(z)));
      }
      any_out = 1;
      c_out++;
      out_h |= 1 << r;
    }
    if (st->act)
      st->act[(size_t)L * NK + kh] = qa | (ka << 1) | (anyg_h << 2) | (out_h << 8);
  }
  if (st->cnt) {
    st->cnt[LXO_C_CHANS] += n_ch;
    st->cnt[LXO_C_QKV_ENT] += n_ent;
    st->cnt[LXO_C_BA_ENT] += c_ba;
    st->cnt[LXO_C_Z_ENT] += c_z;
    st->cnt[LXO_C_ROWS] += c_rows;
    st->cnt[LXO_C_VH_ACTIVE] += c_act;
    st->cnt[LXO_C_VH_WRITE] += c_wr;
    st->cnt[LXO_C_VH_OUT] += c_out;
  }
  if (!any_out) return;
  // out_proj (bf16 linear) added to the residual in bf16
  int64_t c_oe = 0, c_chg = 0;
#pragma omp parallel for schedule(static) reduction(+ : c_oe, c_chg)
  for (int rr = 0; rr < H; rr++) {
    const lxo_csr* m = &ly->out;
    if (m->indptr[rr + 1] == m->indptr[rr]) continue;
    float s = 0.0f;
    int any = 0;
    for (int64_t e = m->indptr[rr]; e < m->indptr[rr + 1]; e++) {
      const float o = st->on[m->indices[e]];
      if (o != 0.0f) {
        s = lx_add(s, lx_mul(o, lx_f(m->data[e])));
        any = 1;
        c_oe++;
      }
    }
    if (any) {
      const float nx = lx_rbf(lx_add(x[rr], lx_rbf(s)));
      c_chg += nx != x[rr];
      x[rr] = nx;
    }
  }
  if (st->cnt) {
    st->cnt[LXO_C_OUT_ENT] += c_oe;
    st->cnt[LXO_C_GDN_WRITE] += c_oe > 0;
  }
  (void)c_chg;
}

static void mlp_layer(lxo_run* st, int L) {
  const lxo_chip* chip = st->chip;
  const lxo_layer* ly = &chip->layers[L];
  float* x = st->x;
  float* xn = st->xn;
  rms_norm(x, ly->ln_post, chip->eps, xn);
  const int64_t nu = ly->gate.rows;
  float* h = (float*)calloc((size_t)nu, sizeof(float));
  int64_t c_gu = 0, c_dn = 0;
#pragma omp parallel for schedule(static) reduction(+ : c_gu)
  for (int64_t u = 0; u < nu; u++) {
    if (ly->gate.indptr[u + 1] == ly->gate.indptr[u] || ly->up.indptr[u + 1] == ly->up.indptr[u])
      continue;
    c_gu += ly->gate.indptr[u + 1] - ly->gate.indptr[u] + ly->up.indptr[u + 1] - ly->up.indptr[u];
    // down_proj(silu(gate(x)) * up(x)), every product of bf16 tensors rounded to bf16
    const float gg = lx_rbf(row_dot(&ly->gate, u, xn));
    const float uu = lx_rbf(row_dot(&ly->up, u, xn));
    const float act = lx_rbf(lx_silu(gg));
    h[u] = lx_rbf(lx_mul(act, uu));
  }
#pragma omp parallel for schedule(static) reduction(+ : c_dn)
  for (int rr = 0; rr < H; rr++) {
    const lxo_csr* m = &ly->down;
    float s = 0.0f;
    int any = 0;
    for (int64_t e = m->indptr[rr]; e < m->indptr[rr + 1]; e++) {
      const float hv = h[m->indices[e]];
      if (hv != 0.0f) {
        s = lx_add(s, lx_mul(hv, lx_f(m->data[e])));
        any = 1;
        c_dn++;
      }
    }
    if (any) x[rr] = lx_rbf(lx_add(x[rr], lx_rbf(s)));
  }
  free(h);
  if (st->cnt) {
    st->cnt[LXO_C_GU_ENT] += c_gu;
    st->cnt[LXO_C_DOWN_ENT] += c_dn;
  }
}

// the head's dense columns (see the header comment); returns their count (0: none)
static int head_dense_cols(const lxo_csr* hd, int* cols) {
  int64_t* cnt = (int64_t*)calloc(H, sizeof(int64_t));
  for (int64_t e = 0; e < hd->indptr[hd->rows]; e++) cnt[hd->indices[e]]++;
  int n = 0;
  for (int c = 0; c < H; c++)
    if (cnt[c] == hd->rows && hd->rows > 0) {
      if (n == 32) {
        n = 33;
        break;
      }
      cols[n++] = c;
    }
  free(cnt);
  if (n == 0 || n > 32) return 0;
  float vals[4];
  int nv = 0;
  for (int64_t r = 0; r < hd->rows; r++) {
    for (int64_t e = hd->indptr[r]; e < hd->indptr[r + 1]; e++) {
      int dense = 0;
      for (int i = 0; i < n; i++) dense |= hd->indices[e] == cols[i];
      if (!dense) continue;
      const float v = lx_f(hd->data[e]);
      int seen = 0;
      for (int i = 0; i < nv; i++) seen |= vals[i] == v;
      if (!seen) {
        if (nv == 4) return 0;
        vals[nv++] = v;
      }
    }
  }
  return n;
}

static int head_argmax(lxo_run* st, float* margin_out) {
  const lxo_chip* chip = st->chip;
  const lxo_csr* hd = &chip->head;
  float xf[H];
  rms_norm(st->x, chip->final_norm, chip->eps, xf);
  enum { NCH = 64 };  // row chunks, combined in row order (the first maximum wins)
  float cb[NCH], cs[NCH];
  int ci[NCH];
  const int64_t V = hd->rows;
#pragma omp parallel for schedule(static)
  for (int k = 0; k < NCH; k++) {
    float best = -LXB_INF, second = -LXB_INF;
    int bi = -1;
    for (int64_t t = V * k / NCH; t < V * (k + 1) / NCH; t++) {
      float D = 0.0f, S = 0.0f;
      int di = 0;
      float grp = 0.0f;
      int in_grp = 0;
      for (int64_t e = hd->indptr[t]; e < hd->indptr[t + 1]; e++) {
        const int c = hd->indices[e];
        const float p = lx_mul(lx_f(hd->data[e]), xf[c]);
        if (di < st->n_dense && st->dense_cols[di] == c) {
          grp = lx_add(grp, p);
          di++;
          if (++in_grp == 4 || di == st->n_dense) {
            D = lx_add(D, grp);
            grp = 0.0f;
            in_grp = 0;
          }
        } else {
          S = lx_add(S, p);
        }
      }
      const float lg = lx_rbf(lx_add(D, S));
      if (bi < 0 || lg > best) {  // the first maximum: a later equal logit does not replace it
        second = bi < 0 ? -LXB_INF : best;
        best = lg;
        bi = (int)t;
      } else if (lg > second) {
        second = lg;
      }
    }
    cb[k] = best;
    cs[k] = second;
    ci[k] = bi;
  }
  int w = -1;
  for (int k = 0; k < NCH; k++)
    if (ci[k] >= 0 && (w < 0 || cb[k] > cb[w])) w = k;
  float second = -LXB_INF;
  for (int k = 0; k < NCH; k++) {
    if (ci[k] < 0) continue;
    if (cs[k] > second) second = cs[k];
    if (k != w && cb[k] > second) second = cb[k];
  }
  if (margin_out) *margin_out = lx_sub(cb[w], second);
  if (st->cnt) {  // 8 bytes of codes per row; 4 per sparse entry whose column's input is nonzero
    unsigned char dense[H];  // (the others add zeros: a kernel may skip them)
    memset(dense, 0, sizeof(dense));
    for (int j = 0; j < st->n_dense; j++) dense[st->dense_cols[j]] = 1;
    int64_t sp = 0;
    for (int64_t e = 0; e < hd->indptr[V]; e++) {
      const int c = hd->indices[e];
      sp += !dense[c] && xf[c] != 0.0f;
    }
    st->cnt[LXO_C_HEAD_B] += (st->n_dense ? 8 * V : 0) + 4 * sp;
  }
  return ci[w];
}

// n_tokens steps of the model alone: step i embeds forced[i] (i < n_forced) or step i-1's
// prediction. rec and conv are updated in place. preds[i] is step i's argmax; inputs (if set)
// each step's input; margins (if set) each step's top-2 logit margin; resid (if set) the
// residual after the chip layers at each step, [n_tokens][H] fp32. Returns 0, or -1 on a bad
// token id.
int lxo_decode(const lxo_chip* chip, float* rec, uint16_t* conv, const int32_t* forced,
               int n_forced, int n_tokens, int32_t* preds, int32_t* inputs, float* margins,
               float* resid, int64_t* counts, float* xin, int32_t* act) {
  lxo_run* st = (lxo_run*)calloc(1, sizeof(lxo_run));
  st->chip = chip;
  st->rec = rec;
  st->conv = conv;
  st->n_dense = head_dense_cols(&chip->head, st->dense_cols);
  int tok = forced[0];
  int rc = 0;
  for (int i = 0; i < n_tokens; i++) {
    if (i < n_forced) tok = forced[i];
    if (tok < 0 || (int64_t)tok + chip->offset >= chip->n_embed) {
      rc = -1;
      break;
    }
    if (inputs) inputs[i] = tok;
    st->cnt = counts ? counts + (size_t)i * LXO_C_N : NULL;
    st->xin = xin ? xin + (size_t)i * chip->n_layers * H : NULL;
    st->act = act ? act + (size_t)i * chip->n_layers * NK : NULL;
    const uint16_t* e = chip->embed + ((int64_t)tok + chip->offset) * H;
    for (int c = 0; c < H; c++) st->x[c] = lx_f(e[c]);
    for (int L = 0; L < chip->n_layers; L++) {
      gdn_layer(st, L);
      mlp_layer(st, L);
    }
    if (resid) memcpy(resid + (size_t)i * H, st->x, sizeof(float) * H);
    const int p = head_argmax(st, margins ? margins + i : NULL);
    preds[i] = p;
    tok = p;
  }
  free(st);
  return rc;
}

// the canonical sums, exposed for the kernels' unit tests
int lxo_n_counters(void) { return LXO_C_N; }
float lxo_ssq2560(const float* x) { return ssq2560(x); }
float lxo_sumsq128(const float* x) { return sumsq128(x); }
void lxo_l2norm_bf16(const float* x, int n, float* out) { l2norm_bf16(x, n, out); }
float lxo_exp(float x) { return lx_exp(x); }
float lxo_log1p(float x) { return lx_log1p(x); }
float lxo_silu(float x) { return lx_silu(x); }
float lxo_sigmoid(float x) { return lx_sigmoid(x); }
float lxo_softplus(float x) { return lx_softplus(x); }
