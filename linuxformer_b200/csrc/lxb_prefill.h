// The prefill plan image: the weight tables of the chunked-prefill kernels (prefill.cu), packed
// by linuxformer_b200/prefill_tables.py into one byte image that lxb_prefill_plan_create
// validates and uploads whole. Offsets are byte offsets from the image start (sections) or
// element indices into a section; all fields are 4- or 8-byte little-endian.
//
// These tables restate what the reference's sparse prefill finds per layer (lx/lx/fast.py:187-248:
// the live rows and columns of every projection) for a token-parallel layout: every stage of a
// layer runs over the whole chunk, one thread per token (or per value-head column for the
// recurrence), so a table row is read once per block of tokens.
//   - tap channels: the in_proj_qkv channels with a nonzero conv tap (the only ones whose conv
//     output can be nonzero), each with its in_proj_qkv row;
//   - live key heads: those with a query or key tap channel; their live rows (at most
//     LXB_PF_MAXLIVE) are the only recurrent-state rows a query or key ever reaches, so the
//     recurrence keeps exactly those rows of each value head in registers, and every other row
//     of the state only decays;
//   - out_proj rows over the live value heads' dims (another head's output is exactly 0);
//   - MLP units with nonzero gate and up rows and a down column, and down_proj rows over them;
//   - the head: its dense columns as 2-bit codes (as the decode plan) and the rest as CSR rows.
#pragma once
#include <stdint.h>

#define LXB_PF_MAGIC 0x46505a4cu  // "LZPF"
#define LXB_PF_VERSION 1
#define LXB_PF_MAXLIVE 31         // live query/key rows per key head (bit 31 of a mask: any)
#define LXB_PF_MAXDENSE 32

enum {
  LXB_PF_SEC_LAYERS = 0,  // lxb_pf_layer[n_layers]
  LXB_PF_SEC_ENT,         // uint32 entries: low 16 bits an index, high 16 bits a bf16 weight
  LXB_PF_SEC_I32,         // int32 pool
  LXB_PF_SEC_U16,         // uint16 pool: bf16 parameters
  LXB_PF_SEC_TAPS,        // lxb_pf_tap[]
  LXB_PF_SEC_VHS,         // lxb_pf_vh[n_layers * 128]
  LXB_PF_SEC_UNITS,       // lxb_pf_unit[]
  LXB_PF_SEC_HCODES,      // uint64 per vocabulary row: the dense columns' 2-bit codes
  LXB_PF_SEC_COUNT
};

typedef struct {
  int64_t off;    // bytes from the image start (16-aligned)
  int64_t count;  // elements
} lxb_pf_sec;

typedef struct {
  uint32_t magic, version;
  int32_t n_layers, n_vocab;
  int32_t hidden, n_dense;
  int64_t n_embed_rows;  // rows the embedding must have
  int32_t offset;        // chip token t embeds row offset + t
  float eps;             // rms_norm_eps (every RMSNorm and the gated norm)
  int32_t final_norm;    // u16 pool offset of the final norm weight [2560]
  int32_t head_ptr;      // i32 pool: n_vocab + 1 entry pointers of the head's sparse entries
  float htab[4];         // the dense head columns' values, by code
  int32_t dense_cols[LXB_PF_MAXDENSE];
  int32_t max_tap, max_lvh;     // the largest per-layer tap-channel and live-value-head counts
  int32_t max_slot, max_units;  // ... live slots and MLP units
  lxb_pf_sec sec[LXB_PF_SEC_COUNT];
} lxb_pf_header;

typedef struct {
  int32_t ln_in, ln_post;  // u16 pool offsets of input_layernorm / post_attention_layernorm
  int32_t gnorm;           // u16 pool offset of the gated norm's weight [128]
  int32_t tap0, n_tap;     // taps[tap0, tap0 + n_tap)
  int32_t chan;            // i32 pool: per conv channel (24576): tap index or -1, entry offset,
                           // entry count (its in_proj_qkv row; for its conv window)
  int32_t khs, n_kh;       // i32 pool: per live key head: key head, first slot, live rows
  int32_t slots, n_slot;   // i32 pool: per slot: state row, query tap or -1, key tap or -1
                           // (a live key head's slots in ascending row order)
  int32_t livemask;        // i32 pool: per key head (16) 8 words, bit r: row r is a live row
  int32_t vtap;            // i32 pool: per live value dim (n_kh * 1024): its value tap or -1
  int32_t zrow;            // i32 pool: per live value dim: (entry offset, count) of in_proj_z
  int32_t out_ptr;         // i32 pool: 2561 entry pointers of out_proj rows (index: live dim)
  int32_t unit0, n_units;  // units[unit0, unit0 + n_units)
  int32_t down_ptr;        // i32 pool: 2561 entry pointers of down_proj rows (index: unit)
  int32_t nl;              // the most live rows of a key head in this layer (<= LXB_PF_MAXLIVE)
  int32_t pad[2];
} lxb_pf_layer;  // 80 bytes

typedef struct {
  uint32_t ent, n;         // the channel's in_proj_qkv entries (column | bf16 << 16)
  uint32_t conv_ch;        // its index in the layer's conv state
  uint32_t t01, t23;       // conv taps 0..3, bf16 pairs (low half first)
  uint32_t pad[3];
} lxb_pf_tap;  // 32 bytes

typedef struct {
  uint32_t a_ent, a_n;     // in_proj_a row
  uint32_t b_ent, b_n;     // in_proj_b row
  uint16_t A_log, dt_bias; // bf16
  uint32_t pad[3];
} lxb_pf_vh;  // 32 bytes

typedef struct {
  uint32_t g, u;           // gate / up row entries: the up entries follow the gate entries
  uint32_t ng, nu;         // (u == g + ng), so a unit's two rows are one list
} lxb_pf_unit;  // 16 bytes

#ifdef __cplusplus
static_assert(sizeof(lxb_pf_layer) == 80 && sizeof(lxb_pf_tap) == 32, "prefill layout");
static_assert(sizeof(lxb_pf_vh) == 32 && sizeof(lxb_pf_unit) == 16, "prefill layout");
static_assert(sizeof(lxb_pf_header) == 336, "prefill header layout");
#endif
