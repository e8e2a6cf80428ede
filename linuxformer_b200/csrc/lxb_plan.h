// The plan image: every weight table the decode kernel reads, packed by
// linuxformer_b200/tables.py into one byte image that lxb_plan_create validates and uploads
// whole. All offsets are byte offsets from the image start (sections) or element indices into
// a section; all structs are plain 4/8-byte fields, little-endian, no padding surprises.
//
// The tables restate what the reference packs in lx/lx/mega.py:199-504 (its CSR rows, the CSC
// of out_proj/down_proj, per-item channel lists, the head's dense codes and sparse columns), laid
// out for a thread-block cluster per stream instead of one persistent grid:
//   - a GDN item (one live key head of one layer) runs on one CTA of the cluster;
//   - the residual rows are split in C contiguous blocks of 2560 / C; the CTA owning a block
//     computes every sum that lands in it (down_proj and out_proj rows, in CSR order), so no
//     sum is ever split across CTAs and none needs an atomic;
//   - the head's rows are split in C contiguous ranges.
#pragma once
#include <stdint.h>

#define LXB_MAGIC 0x50425a4cu  // "LZBP"
#define LXB_IMAGE_VERSION 10

#define LXB_H 2560
#define LXB_KD 256
#define LXB_VD 128
#define LXB_NK 16
#define LXB_NV 128
#define LXB_R 8
#define LXB_CONV 24576
#define LXB_NSLOT 1536  // an item's q | k | v: q 0..255, k 256..511, v 512 + r * 128 + j
#define LXB_NOSLOT 0xffffu
#define LXB_MAXC 16     // CTAs per cluster
#define LXB_MINC 4
#define LXB_ITEMSLOTS 4 // items one CTA may run in one layer
#define LXB_HEADSLICES 32  // the head's rows in this many slices per CTA rank (helper clusters)
#define LXB_HEADMAIN 2     // of which the decoding cluster takes the first (it also gathers)
#define LXB_MAXDENSE 32
#define LXB_MAXUNITS 2048  // MLP units one CTA evaluates in one layer
#define LXB_MAXWIN 1024    // query/key conv windows one CTA keeps in shared memory for a launch
#define LXB_NOWIN 0xffffffffu

// item flags
#define LXB_IT_DECAYS 1  // some value head's g may be nonzero
#define LXB_IT_OUT 2     // the key head's value dims have out_proj entries
#define LXB_IT_NONRES 4  // some query/key window is not resident in shared memory (its CTA's
                         // window table was full): the item never runs speculatively

enum {
  LXB_SEC_LAYERS = 0,  // lxb_layer[n_layers]
  LXB_SEC_ITEMS,       // lxb_item[n_items]
  LXB_SEC_CHANS,       // lxb_chan[]
  LXB_SEC_ENT,         // uint32 entries: low 16 bits an index, high 16 bits a bf16 weight
  LXB_SEC_UNITS,       // lxb_unit[]
  LXB_SEC_OWNERS,      // lxb_owner[n_layers * cluster]
  LXB_SEC_I32,         // int32 pool: row pointers, row refs, item-of tables
  LXB_SEC_U16,         // uint16 pool: bf16 parameters (norm weights, A_log, dt_bias, gated norm)
  LXB_SEC_HEADCTA,     // lxb_headcta[(LXB_HEADSLICES + 1) * cluster]: slice k of rank c at
                       // c * LXB_HEADSLICES + k, then the ranks' whole ranges
  LXB_SEC_HCODES,      // uint64 per vocabulary row: the dense columns' 2-bit codes
  LXB_SEC_BLOBS,       // bytes: the step blobs (below)
  LXB_SEC_BLOBIDX,     // lxb_blobref[(n_layers + 1) * cluster]: layer L (or the head, L =
                       // n_layers) of CTA c at L * cluster + c
  LXB_SEC_WINMAP,      // int32 (layer, conv channel) pairs: the windows each CTA keeps resident
  LXB_SEC_WINIDX,      // int32 (offset in pairs, count) per CTA into WINMAP
  LXB_SEC_COUNT
};

typedef struct {
  int64_t off;    // bytes from the image start (16-aligned)
  int64_t count;  // elements
} lxb_sec;

typedef struct {
  uint32_t magic, version;
  int32_t n_layers, cluster;
  int32_t n_vocab, hidden;
  int32_t n_items, n_dense;
  int64_t n_embed_rows;  // rows the embedding must have
  int32_t offset;        // chip token t embeds row offset + t
  float eps;             // rms_norm_eps (every RMSNorm and the gated norm)
  int32_t final_norm;    // u16 pool offset of the final norm weight [2560]
  int32_t pad0;
  float htab[4];         // the dense head columns' values, by code
  int32_t dense_cols[LXB_MAXDENSE];
  int32_t blob_max;      // the largest step blob, bytes
  int32_t hsp_mask;      // i32 pool offset: 80 words, bit c set if head column c has sparse
                         // entries (-1: none)
  int32_t pad1[2];
  lxb_sec sec[LXB_SEC_COUNT];
} lxb_image_header;

typedef struct {
  int32_t has_gdn, has_mlp;
  int32_t ln_in, ln_post;  // u16 pool offsets of input_layernorm / post_attention_layernorm [2560]
  int32_t item0, n_items;  // items [item0, item0 + n_items)
  int32_t owner0;          // owners[owner0 + rank]
  int32_t itemof;          // i32 pool offset: item index of key head kh (16 entries, -1 none)
  int32_t decays;          // some item of the layer decays (its bitmaps are kept)
  int32_t mrow0, mrow1;    // the rows the MLP can change, [mrow0, mrow1): the owners' MLP row
                           // ranges tile it in rank order (both 0 without an MLP)
  int32_t pad;
} lxb_layer;  // 48 bytes

typedef struct {
  int32_t layer, kh, cta, slot;
  int32_t ch0, n_ch;       // chans[ch0, ch0 + n_ch)
  int32_t rows;            // i32 pool: (entry offset, count) pairs: 8 beta, 8 a, 1024 z rows
  int32_t params;          // u16 pool: A_log[8], dt_bias[8], gated-norm weight[128]
  int32_t flags;           // LXB_IT_*
  int32_t n_eager;         // chans [ch0, ch0 + n_eager): query/key channels with a nonzero tap,
                           // evaluated every step
  int32_t n_vneed;         // then value channels with a nonzero tap: evaluated on the steps a key
                           // fires; every channel from n_eager on keeps its conv window lazily
                           // (recomputed from the residual ring at the launch's end)
  int32_t tapu;            // the union of the value channels' tap masks (bit p: tap p nonzero)
} lxb_item;  // 48 bytes

typedef struct {
  uint32_t ent;            // entries [ent, ent + n): column | bf16 << 16
  uint16_t n, slot;        // entry count; place in q | k | v (LXB_NOSLOT: window only)
  uint32_t conv_ch;        // the channel's index in the layer's conv state
  uint32_t t01, t23;       // conv taps 0..3, bf16 pairs (low half first)
  uint32_t tapmask;        // bit j: tap j is nonzero
  uint32_t win;            // a query/key channel's resident window slot in its CTA's shared
                           // memory (as its blob entry's), else LXB_NOWIN
  uint32_t pad;
} lxb_chan;  // 32 bytes: two aligned 16-byte loads

typedef struct {
  uint32_t g, u;           // gate / up row entries
  uint16_t ng, nu;
  uint32_t pad;
} lxb_unit;  // 16 bytes

typedef struct {
  int32_t mr0, mr1;        // the MLP rows this CTA owns, [mr0, mr1): multiples of 8, at most
                           // H / LXB_MINC rows (the out_proj rows are rank * blk .. + blk)
  int32_t nlong;           // owned out_proj rows with more than LXB_LONG entries (by warps)
  int32_t orow;            // i32 pool: blk + 1 entry pointers of the owned rows' out_proj
                           // entries (value dim | bf16 << 16), or -1
} lxb_owner;  // 16 bytes

typedef struct {
  int32_t r0, r1;          // head rows [r0, r1)
  int32_t rowptr;          // i32 pool: r1 - r0 + 1 entry pointers (the rows' sparse entries)
  int32_t pad;
} lxb_headcta;  // 16 bytes

// --- step blobs ---------------------------------------------------------------------------------
// Everything one CTA reads on one step of the token loop, packed contiguously so that a single
// stream of bulk copies (cp.async.bulk, TMA) brings it into shared memory one step ahead: the
// layer's norm weights, the CTA's GDN items (their query/key channels with the in_proj
// entries, the beta/a rows, the per-head parameters) and the MLP units its residual rows need
// (gate/up entries, the rows' down_proj entries). Offsets are bytes from the blob's start, all
// 16-aligned; entries are uint32 (index | bf16 << 16). The head's blob holds the final norm.
typedef struct {
  int64_t off;             // bytes from the BLOBS section start (16-aligned)
  int32_t bytes;           // a multiple of 16
  int32_t pad;
} lxb_blobref;

typedef struct {
  int32_t bytes, n_items;
  int32_t item[LXB_ITEMSLOTS];  // offsets of lxb_bitem
  int32_t ln_in, ln_post;       // offsets of bf16[2560] norm weights, or -1
  int32_t mlp;                  // offset of lxb_bmlp, or -1
  int32_t pad[7];
} lxb_bhdr;  // 64 bytes

typedef struct {
  int32_t item;            // the global item (lazy channels, z rows, output flags)
  int32_t n_eager, eager;  // n_eager lxb_bchan at offset eager
  int32_t rows;            // 16 int32 pairs (entry offset in bytes, count): 8 beta, 8 a rows
  int32_t prm;             // bf16 A_log[8], dt_bias[8], gated-norm weight[128]
  int32_t kh, slot, flags; // as the global item's
  int32_t z;               // offset of int32 zptr[1025] (entry indices) then the in_proj_z
                           // entries of the head's 1024 value dims; -1: no output possible
  int32_t pad[7];
} lxb_bitem;  // 64 bytes

typedef struct {
  int32_t ent;             // byte offset of its entries
  uint16_t n, slot;
  uint32_t conv_ch, t01, t23;
  uint32_t win;            // its window's resident slot (LXB_NOWIN: read in global memory)
  uint32_t pad[2];
} lxb_bchan;  // 32 bytes

typedef struct {
  int32_t n_units, units;  // n_units lxb_bunit at offset units
  int32_t down_ptr;        // int32[nr + 1]: the owned rows' entries (indices into down_ent)
  int32_t down_ent;        // uint32 entries: local unit | bf16 << 16
  int32_t r0, nr;          // the owned MLP rows [r0, r0 + nr): the owner's mr0, mr1 - mr0
  int32_t nlong;           // of them, rows with more than LXB_LONG entries (summed by warps)
  int32_t pad;
} lxb_bmlp;  // 32 bytes

typedef struct {
  int32_t g, u;            // byte offsets of the gate / up entries
  uint16_t ng, nu;
  int32_t pad;
} lxb_bunit;  // 16 bytes

#ifdef __cplusplus
static_assert(sizeof(lxb_bhdr) == 64 && sizeof(lxb_bitem) == 64 && sizeof(lxb_bchan) == 32,
              "blob layout");
static_assert(sizeof(lxb_bmlp) == 32 && sizeof(lxb_bunit) == 16 && sizeof(lxb_blobref) == 16,
              "blob layout");
static_assert(sizeof(lxb_image_header) == 440, "lxb_image_header layout");
static_assert(sizeof(lxb_layer) == 48 && sizeof(lxb_item) == 48, "layer/item layout");
static_assert(sizeof(lxb_chan) == 32 && sizeof(lxb_unit) == 16, "chan/unit layout");
static_assert(sizeof(lxb_owner) == 16 && sizeof(lxb_headcta) == 16, "owner/headcta layout");
#endif
