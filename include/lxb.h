/* linuxformer-b200: the C ABI of the sparse chip decode (B200, sm_100a).
 *
 * One shared library, liblxb.so, replaces the reference's megakernel boundary: the ctypes
 * interface of lx/csrc/mega.cu (mk_run, mk_smem_base, mk_max_ctas, mk_max_smem,
 * mk_last_error: mega.cu:864-893), which lx/lx/mega.py loads through lx/lx/mk_build.py:40-57.
 * Plain pointers and sizes only; every call returns 0 or an error code (a positive cudaError
 * value, or a negative LXB_E_* value); nothing throws across the boundary. Launches are
 * asynchronous on the stream given. A plan is not thread-safe: one launch at a time per plan.
 *
 * Buffer ownership follows the reference (lx/lx/mega.py:506-574): the caller owns the machine
 * state (HF cache layout: recurrent [128][256][128] fp32 and conv [24576][4] bf16 per layer,
 * updated in place), the embedding, and the forced/preds/inputs arrays; the plan owns the
 * weight tables it uploads.
 */
#ifndef LXB_ABI_H_
#define LXB_ABI_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LXB_ABI_VERSION 1

/* error codes (negative; positive values are cudaError_t) */
#define LXB_OK 0
#define LXB_E_INVAL (-1)     /* a bad argument */
#define LXB_E_IMAGE (-2)     /* a malformed plan image (an offset, count or index out of range) */
#define LXB_E_DEVICE (-3)    /* the device cannot run the plan (arch, cluster size, shared memory) */
#define LXB_E_STATUS (-4)    /* the kernel reported an error: read it with lxb_status */
#define LXB_E_TOOBIG (-5)    /* more scratch than lxb_decode_noalloc's fixed array holds */

/* lxb_decode_noalloc's scratch: a fixed device array of this many bytes per GPU */
#define LXB_NOALLOC_MAX_SCRATCH (4u << 20)
#define LXB_MAX_DEVICES 64

/* device status bits (lxb_status) */
#define LXB_S_TOKEN 1u       /* a token id outside the embedding: clamped, the stream is invalid */
#define LXB_S_STAGE 2u       /* a staging copy did not land within 2 s: later steps skipped */
#define LXB_S_HELPER 4u      /* a head helper cluster did not answer in time: the decoding cluster
                                took its rows itself (informational: the stream is exact) */
#define LXB_S_SYNC 8u        /* a grid barrier of the text decode did not complete within 2 s: the
                                launch stopped early, its results are invalid */

typedef struct lxb_plan lxb_plan;

typedef struct {
  int device;
  int cc_major, cc_minor;
  int sm_count;
  int max_smem_optin;   /* bytes per block */
  int cluster_launch;   /* cudaDevAttrClusterLaunch */
  int max_clusters;     /* co-resident clusters of the plan's size (0 before a plan exists) */
} lxb_caps;

typedef struct {
  uint32_t status;      /* LXB_S_* bits, sticky until lxb_status_clear */
  int32_t first_stream; /* the first stream that set a bit */
  int32_t first_step;
} lxb_error;

/* ABI version of the library (LXB_ABI_VERSION). Replaces nothing: the reference's ctypes loader
 * trusted the .so it had just compiled (lx/lx/mk_build.py:40-57). */
int lxb_abi_version(void);

/* Device capabilities. Replaces mk_max_smem / mk_max_ctas (mega.cu:876-890). */
int lxb_query(int device, lxb_caps* caps);

/* Upload a plan image (the packed weight tables, format in lxb_plan.h, built by
 * linuxformer_b200.tables) to the current device, validating every offset and index. cluster is
 * the number of CTAs that run one stream (8 or 16). Replaces Mega.__init__'s uploads
 * (lx/lx/mega.py:458-504) and the launch setup of mk_run (mega.cu:867-874). */
int lxb_plan_create(const void* image, size_t bytes, int cluster, lxb_plan** out);

/* Decode n_tokens steps of n_streams independent machines (one thread-block cluster each).
 * Stream s: step i embeds forced[s * n_forced + i] for i < n_forced, else its own step i-1
 * prediction; preds[s * n_tokens + i] receives step i's argmax, inputs (optional, may be NULL)
 * the token each step embedded. state_ptrs: a DEVICE array of n_streams * n_layers * 2 uint64,
 * (recurrent, conv) device pointers per stream and layer. bitmaps: a DEVICE array of
 * n_streams * n_layers * 128 * 8 uint32, the nonzero-row bitmaps of the recurrent states; with
 * sync_bitmaps != 0 they are rebuilt from the states first (the reference's sync_bitmaps,
 * mega.py:518-526). embed: DEVICE bf16 [n_embed_rows][2560]; token t embeds row offset + t.
 * Replaces mk_run (mega.cu:867-874) as called by Mega.run (mega.py:529-574). */
int lxb_decode(lxb_plan* plan, const uint64_t* state_ptrs, uint32_t* bitmaps, int sync_bitmaps,
               void* scratch, const uint16_t* embed, int n_streams, const int32_t* forced,
               int n_forced, int n_tokens, int32_t* preds, int32_t* inputs, void* cuda_stream);

/* Device scratch lxb_decode needs for n_streams streams (a ring of the last 4 steps' residual
 * rows per layer, from which the lazily kept conv windows are recomputed, and the head helpers'
 * exchange area). The caller allocates it (16-byte aligned) and need not initialise it: the
 * launch clears, on its stream, the words that must start cleared. Its contents do not outlive a
 * call, so one buffer may serve several plans in turn, but not two launches at once. */
size_t lxb_scratch_bytes(const lxb_plan* plan, int n_streams);

/* lxb_decode for callers that cannot allocate device memory. No counterpart in the reference
 * (its Python host allocates freely). Some hosts cannot hand this library device memory once
 * they are running: a server that carves all device memory into one pool at start-up, or a
 * host whose allocator is not CUDA-aware and only passes the buffers it owns (state, tokens,
 * predictions). This call takes the same arguments as lxb_decode except the scratch, which it
 * takes from a fixed array inside the library (LXB_NOALLOC_MAX_SCRATCH bytes, held by every GPU
 * that loads the library until the process exits): it calls no cudaMalloc or cudaFree.
 * Requests needing more (lxb_scratch_bytes(plan, n_streams) above the limit; for the 37-layer
 * chip about 5 streams) return LXB_E_TOOBIG. The first call on a device looks up the array's
 * device address there (the device must be current); make that first call before any stream
 * capture. All calls on a device share the array: calls that overlap on the GPU race. */
int lxb_decode_noalloc(lxb_plan* plan, const uint64_t* state_ptrs, uint32_t* bitmaps,
                       int sync_bitmaps, const uint16_t* embed, int n_streams,
                       const int32_t* forced, int n_forced, int n_tokens, int32_t* preds,
                       int32_t* inputs, void* cuda_stream);

/* The device status word (after the stream has synchronised). Replaces mk_last_error
 * (mega.cu:892) for kernel-side errors. */
int lxb_status(lxb_plan* plan, lxb_error* err);
int lxb_status_clear(lxb_plan* plan);

/* Per-section cycle counters (the reference's Mega.run(prof=...), lx/csrc/mega.cu:717-737):
 * with a DEVICE buffer of n_streams * cluster * lxb_profile_sections() uint64, every later
 * lxb_decode adds, per stream and CTA, the clock64 cycles spent in each section (norms, GDN
 * items, MLP, barrier, pull, write fix-ups, head, embedding) and two counts (fix-up steps,
 * tokens). NULL turns it off (the default). */
int lxb_plan_set_profile(lxb_plan* plan, unsigned long long* prof);
int lxb_profile_sections(void);

/* An empty cluster barrier's latency in SM clock cycles (one cluster of `cluster` CTAs doing
 * `iters` barriers and nothing else): with the profile's barrier count per token, the decode's
 * barrier floor. Synchronises the device. */
int lxb_cluster_sync_cycles(int cluster, int iters, double* cycles_per_barrier);

/* The device typing queue (no counterpart in the reference's kernel: its host types a command into
 * the model-alone machine between launches, Linux.run_alone, lx/lx/linux.py:254-289). With it
 * set, every later lxb_decode types each stream's queued bytes itself, after any token: a batch of
 * at most rx_slots bytes (the first as key0_base + byte, the others as key_base + byte) replaces
 * the model's prediction as the next input once the current input is a record boundary and the
 * machine has read every byte typed so far. The RX FIFO count is kept per token: an input of
 * class LXB_T_TYPED adds one, an input of class LXB_T_RX takes one away. tstate holds, per
 * stream, the bytes typed, the FIFO count, the bytes left in the current batch and the input
 * after the launch's last step; the launch reads it first and writes it last, so the next
 * launch takes &tstate[s * 4 + 3] as its forced first input. NULL (or keys NULL) turns it off. */
#define LXB_T_FINAL 1u  /* a record boundary: a batch may follow this input */
#define LXB_T_TYPED 2u  /* a typed key (enters the RX FIFO) */
#define LXB_T_RX 4u     /* the machine reads a byte (leaves the RX FIFO) */
typedef struct {
  const int32_t* keys;    /* DEVICE [n_streams][max_keys]: the bytes to type */
  const int32_t* n_keys;  /* DEVICE [n_streams]: bytes queued per stream */
  int32_t max_keys;
  int32_t key0_base, key_base;  /* token of a batch's first byte: key0_base + byte; others: key_base + byte */
  int32_t rx_slots;       /* bytes per batch */
  const uint8_t* tclass;  /* DEVICE [n_class]: LXB_T_* bits per token */
  int32_t n_class;
  int32_t* tstate;        /* DEVICE [n_streams][4], zeroed before the first launch */
} lxb_typing;
int lxb_plan_set_typing(lxb_plan* plan, const lxb_typing* typing);

/* Head helpers: a single-stream launch also starts up to this many more clusters (default 7,
 * at most what the device holds beside the decoding cluster), each of which takes a slice of the
 * output head's rows per token and hands its maximum back through the scratch buffer, so the
 * head's table lookups run on up to 8x the SMs. 0 turns them off. A helper that does not answer
 * within a bounded wait is dropped for the rest of the launch (LXB_S_HELPER); the results do not
 * depend on it. A negative count -n is a drill: n helper clusters start but never answer, so the
 * decoding cluster's wait runs out (about 34 ms) and it takes their rows itself (for tests of the
 * fallback). No counterpart in the reference (its head runs on its one 132-CTA grid). */
int lxb_plan_set_head_helpers(lxb_plan* plan, int max_clusters);

/* How the plan stages its per-step tables: buffers (2 = the next step's copy overlaps the
 * current step), bytes per buffer, and the shared memory each CTA uses. */
int lxb_plan_staging(const lxb_plan* plan, int* nbuf, int* stage_bytes, int* smem_bytes);

/* Bytes of the plan's device tables; the number of co-resident clusters for this plan. */
size_t lxb_plan_bytes(const lxb_plan* plan);
int lxb_plan_max_clusters(const lxb_plan* plan);

void lxb_plan_destroy(lxb_plan* plan);

/* --- The chunked prefill (verified mode) -----------------------------------------------------
 *
 * The reference checks a proposed trace by running it as chunked prefill: Session.verify
 * (lx/lx/session.py:86-116) embeds each chunk and calls Fast.forward (lx/lx/fast.py:252-257) and
 * Fast.head_argmax (fast.py:544-550), then compares every position's argmax with the next token.
 * A prefill plan holds the chip's tables in a token-parallel layout (format in
 * linuxformer_b200/csrc/lxb_prefill.h, built by linuxformer_b200.prefill_tables); one call runs one
 * chunk of T tokens through every chip layer, updating the caller's state in place (the HF cache
 * layout, as lxb_decode), with the same results as T single-token decode steps with every input
 * forced: predictions, conv windows and recurrent states bit for bit. Calls are asynchronous on the
 * given stream (the plan also runs work on a stream of its own, joined back before the call's last
 * operation); the plan's device must be current; one call at a time per plan. */
typedef struct lxb_prefill_plan lxb_prefill_plan;
#define LXB_PF_MAX_T (1 << 23)  /* tokens per call at most (8,388,608) */

/* Validate a prefill image on the host (every offset, count and index); 0 or LXB_E_IMAGE. */
int lxb_prefill_check_image(const void* image, size_t bytes);

/* Validate and upload a prefill image to the current device. Replaces Fast.__init__'s packing of
 * the live rows and columns (lx/lx/fast.py:172-248). LXB_E_IMAGE for a malformed image,
 * LXB_E_DEVICE below compute capability 10. */
int lxb_prefill_plan_create(const void* image, size_t bytes, lxb_prefill_plan** out);

/* Device scratch one call of T tokens needs (the caller allocates it, 256-byte aligned, no
 * initialisation; a call for fewer tokens fits in it). */
size_t lxb_prefill_scratch_bytes(const lxb_prefill_plan* plan, int T);

/* Verify one chunk: embed tokens[0..T) (DEVICE int32; row offset + id of the DEVICE bf16 embedding
 * [rows][2560]), run the chip layers on the state (state_ptrs: a DEVICE array of n_layers * 2
 * uint64, recurrent and conv pointers per layer), write preds[i] (DEVICE int32 [T]) = the head's
 * first argmax at position i, and, if first_wrong (DEVICE int32) is not NULL, the first i < T - 1
 * with preds[i] != tokens[i + 1], or -1. A token id outside the embedding is clamped and reported
 * by lxb_prefill_status (LXB_S_TOKEN). Replaces one chunk of Session.verify
 * (lx/lx/session.py:94-100) with Fast.forward and Fast.head_argmax. */
int lxb_prefill(lxb_prefill_plan* plan, const uint64_t* state_ptrs, const uint16_t* embed,
                const int32_t* tokens, int T, int32_t* preds, int32_t* first_wrong, void* scratch,
                void* cuda_stream);

/* The chip layers alone: h_in (DEVICE bf16 [T][2560], the embedded rows) -> h_out (DEVICE bf16
 * [T][2560], may be NULL or h_in), updating the state. Replaces Fast.forward(h, cache)
 * (lx/lx/fast.py:252-257). */
int lxb_prefill_layers(lxb_prefill_plan* plan, const uint64_t* state_ptrs, const uint16_t* h_in,
                       uint16_t* h_out, int T, void* scratch, void* cuda_stream);

/* The head alone: preds[i] = the first argmax of the head over the final norm of h[i] (DEVICE bf16
 * [T][2560]). Replaces Fast.head_argmax(h) (lx/lx/fast.py:544-550). */
int lxb_prefill_head(lxb_prefill_plan* plan, const uint16_t* h, int T, int32_t* preds,
                     void* scratch, void* cuda_stream);

/* Per-stage timing (the reference's prof counters have no prefill counterpart; its profiler is
 * tools/profile_verify.py over torch.profiler): with timing on, every later call records a CUDA
 * event pair around each kernel launch; lxb_prefill_timing waits for them and returns, per stage
 * kind (index k, named by lxb_prefill_stage_name), the summed milliseconds and the launches since
 * the last read (then clears them). The decay scans run on the plan's second stream beside the
 * others; their time overlaps. */
#define LXB_PF_ROWS 0
#define LXB_PF_NORM 1
#define LXB_PF_TAPS 2
#define LXB_PF_GATES 3
#define LXB_PF_SCAN 4
#define LXB_PF_CONV 5
#define LXB_PF_WINDOWS 6
#define LXB_PF_QK 7
#define LXB_PF_RECUR 8
#define LXB_PF_GNORM 9
#define LXB_PF_OUT 10
#define LXB_PF_MLP 11
#define LXB_PF_DOWN 12
#define LXB_PF_HEAD 13
#define LXB_PF_REDUCE 14
#define LXB_PF_STAGES 15
int lxb_prefill_set_timing(lxb_prefill_plan* plan, int on);
int lxb_prefill_timing(lxb_prefill_plan* plan, double* ms, long long* launches, int n);
const char* lxb_prefill_stage_name(int k);

/* The prefill plan's status word (LXB_S_TOKEN), after the stream has synchronised. */
int lxb_prefill_status(lxb_prefill_plan* plan, lxb_error* err);
int lxb_prefill_status_clear(lxb_prefill_plan* plan);
void lxb_prefill_plan_destroy(lxb_prefill_plan* plan);

/* ---- config 5: the Qwen3.5-4B-shaped text path, batch-1 decode ----------------------------
 * The reference runs its text model (the chip layers merged into Qwen3.5-4B, whose Gated DeltaNet
 * weights are zero-padded to the chip shape, lx/lx/merge.py:82-120) through the stock HF forward
 * (`generate` on merge.text_view, lx/lx/chat.py:62-73, lx/lx/merge.py:251-280); here one
 * persistent cooperative kernel per launch decodes it at batch 1, reading only the non-padding
 * weights (packed by linuxformer_b200/text.py). Layer descriptors hold device addresses: */
typedef struct {
  int32_t type;          /* 0: Gated DeltaNet, 1: gated full attention */
  int32_t flags;         /* LXB_TEXT_GNORM_F32: the gated norm's weight is an fp32 parameter */
  uint64_t w1;           /* input projections, bf16 rows of 2560: GDN q k v z b a (12,352 rows),
                            attention q+gate (per head 256 + 256), k, v (10,240 rows) */
  uint64_t wo;           /* out_proj / o_proj over the live dims: 2560 x 4096 bf16 */
  uint64_t wgu;          /* gate row u, then up row u: 18,432 x 2560 bf16 */
  uint64_t wd;           /* down_proj: 2560 x 9216 bf16 */
  uint64_t ln_in, ln_post;          /* RMSNorm weights [2560] bf16 */
  uint64_t conv_w;       /* GDN: conv taps of the q, k, v channels [8192][4] bf16 */
  uint64_t A_log, dt_bias;          /* GDN: [32] fp32 */
  uint64_t gnorm;        /* GDN: the gated norm's weight [128] as fp32 values */
  uint64_t qn, kn;       /* attention: q_norm / k_norm weights [256] bf16 */
  uint64_t conv_state;   /* GDN: the stock cache's conv windows [24576][4] bf16 (in place) */
  uint64_t rec_state;    /* GDN: the stock cache's recurrent state [128][256][128] fp32 (in place) */
  uint64_t kc, vc;       /* attention: key / value rows [4][max_pos][256] bf16 */
} lxb_text_layer;

/* The gated norm multiplies by its weight in the weight's dtype (Qwen3_5RMSNormGated,
 * modeling_qwen3_5.py:181-190): a bf16 weight rounds the product to bf16, an fp32 one (Qwen's
 * stored dtype, kept by lx/lx/merge.py) does not. */
#define LXB_TEXT_GNORM_F32 1

typedef struct lxb_text_plan_s lxb_text_plan;

/* Copy the layer descriptors to the device and size the launch (one CTA per SM). embed: the
 * embedding [n_embed][2560] bf16; head: the output head [n_vocab][2560] bf16 (the same memory
 * when tied, as Qwen's head is its embedding's first rows, lx/lx/merge.py:251-280); final_norm
 * [2560] bf16; rope: cos and sin of every position, [max_pos][2][64] bf16. LXB_E_INVAL for a
 * null or misaligned address, LXB_E_DEVICE below compute capability 10 or without cooperative
 * launch. */
int lxb_text_plan_create(const lxb_text_layer* layers, int n_layers, const void* embed,
                         int n_embed, const void* head, int n_vocab, const void* final_norm,
                         const void* rope, int max_pos, float eps, int device,
                         lxb_text_plan** out);
size_t lxb_text_scratch_bytes(const lxb_text_plan* plan);
/* n_tokens steps from position pos0 (pos0 + n_tokens <= max_pos): step t's input is forced[t]
 * for t < n_forced, else step t-1's prediction; preds[t] = the first argmax of the head after
 * step t; hidden (or null): [n_tokens][n_layers + 1][2560] fp32, at each step the residual after
 * every layer, then the final norm's output (the stock model's last hidden state). Scratch (lxb_text_scratch_bytes, 256-byte aligned) holds
 * the activations and the grid barrier; it needs no initialisation. Async on the stream. */
int lxb_text_decode(lxb_text_plan* plan, const int32_t* forced, int n_forced, int n_tokens,
                    int pos0, int32_t* preds, float* hidden, void* scratch,
                    size_t scratch_bytes, void* cuda_stream);
int lxb_text_status(lxb_text_plan* plan, uint32_t* status);   /* LXB_S_* bits (synchronises) */
/* Per-section cycle counters of every CTA (the reference's prof counters, lx/csrc/mega.cu:717-737):
 * with a DEVICE buffer of lxb_text_grid(plan) * LXB_TEXT_SECTIONS uint64, every later decode adds,
 * per CTA, the clock64 cycles of each section and the tokens decoded. NULL turns it off. */
#define LXB_TP_NORM 0     /* input vectors: RMSNorms, the gated norm, conv window shifts */
#define LXB_TP_GEMV 1     /* dot products and their epilogues */
#define LXB_TP_WAIT 2     /* waits for a weight chunk to land in shared memory */
#define LXB_TP_SYNC 3     /* grid barriers */
#define LXB_TP_GDN 4      /* the GDN step (conv, norms, gates, delta rule) */
#define LXB_TP_ATT 5      /* attention partials and their combine */
#define LXB_TP_HEAD 6     /* the argmax reduce of the head */
#define LXB_TP_TOKENS 7   /* a count: tokens decoded */
#define LXB_TEXT_SECTIONS 8
int lxb_text_set_profile(lxb_text_plan* plan, unsigned long long* prof);
int lxb_text_status_clear(lxb_text_plan* plan);
int lxb_text_grid(const lxb_text_plan* plan);
void lxb_text_plan_destroy(lxb_text_plan* plan);

/* A short text for an error code. */
const char* lxb_error_string(int code);

#ifdef __cplusplus
}
#endif
#endif /* LXB_ABI_H_ */
