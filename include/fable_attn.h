/*
 * fable_attn.h — C ABI of the B200 (sm_100a) exact-attention engine.
 *
 * This is the boundary the Python layer (fable_attn._C) binds, and the one any other host
 * (ctypes, cgo, JNI, N-API) can bind directly: plain C structs of device pointers, element
 * strides and scalars, no torch types.  Every entry point enqueues work on the caller's CUDA
 * stream and returns without synchronising; the return value is FA_OK (0) or an FA_ERR_* code,
 * with a human-readable message available from fa_last_error().  Nothing here aborts the
 * process.
 *
 * Each parameter block starts with `struct_size`, which the caller sets to sizeof(the struct)
 * it was compiled against; a mismatch is rejected with FA_ERR_ABI instead of reading a
 * differently laid-out block.
 *
 * Counterparts in the reference (MatafakaRespect/flash-attention-rdna2):
 *   fa_forward_launch           <- package/csrc/fa_iface.h:65   (FwdParams, fa_iface.h:10-24)
 *   fable_attn_backward_launch  <- package/csrc/fa_iface.h:66   (BwdParams, fa_iface.h:28-38)
 *   fa_decode_launch            <- package/csrc/fa_iface.h:67-68 (DecParams, fa_iface.h:42-63)
 *   fa_decode_num_splits        <- package/csrc/dispatch.cpp:182-200 (nsplit heuristic)
 *   fa_combine_launch           <- package/fable_attn/flash_attn_interface.py:567-580
 *                                  (flash_attn_combine, torch arithmetic in the reference)
 * The reference passes its structs by value and returns void (aborting on bad input); here they
 * are passed by pointer and the functions return a status code.
 */
#ifndef FABLE_ATTN_H
#define FABLE_ATTN_H

#ifdef __cplusplus
extern "C" {
#endif

#define FA_ABI_VERSION 1

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

/* dtype codes — same numbering as the reference (kernels/fa_forward.hip:403) */
enum { FA_DTYPE_F16 = 0, FA_DTYPE_BF16 = 1, FA_DTYPE_F32 = 2 };

/* status codes */
enum {
  FA_OK = 0,
  FA_ERR_ABI = 1,          /* struct_size mismatch */
  FA_ERR_INVALID = 2,      /* null pointer, bad shape, bad stride */
  FA_ERR_UNSUPPORTED = 3,  /* valid request the engine does not implement (e.g. head_dim) */
  FA_ERR_CUDA = 4,         /* a CUDA runtime/driver call failed */
  FA_ERR_SIZE = 5          /* request exceeds a stated size limit */
};

/* Element strides of a [batch, head, seq, dim] view; the dim stride must be 1. */
typedef struct FaStrides { long long b, h, s; } FaStrides;

/* ------------------------------------------------------------------------------------------
 * Forward (dense and varlen).  Replaces FwdParams / fa_forward_launch.
 *   dense : Q [batch, NH, SQ, HD], K/V [batch, NKV, SK, HD] through the strides (any order of
 *           b/h/s, dim contiguous).  LSE (optional) is written as [batch, NH, SQ] fp32,
 *           natural log.  The reference launches once per batch element
 *           (package/csrc/dispatch.cpp:62-78); here batch is a grid dimension.
 *   varlen: cu_q/cu_k non-null, `batch` = number of sequences, SQ/SK = max_seqlen_q/k (used
 *           only to size the grid), strides.b ignored (token offsets come from cu_*),
 *           seqused_q/k optionally clip each sequence.  LSE (optional) is [NH, lse_total_q].
 * Semantics follow kernels/fa_forward.hip:52-313: s = scale*q.k, softcap c>0 -> c*tanh(s/c),
 * alibi adds slope[h]*(key - q) (signed, no diagonal offset), masks are bottom-right aligned
 * (delta = SK - SQ): causal key > q+delta; window key < q+delta-win_left or
 * key > q+delta+win_right (negative = unbounded); attn_chunk c>0 keeps keys in
 * [floor(max(q+delta,0)/c)*c, +c).  Fully masked rows give O = 0 and LSE = -inf.
 * Dropout: Philox4x32-10 keyed by philox_seed, counter = (h*SQ + q)*SK + key with h the global
 * query head and no batch term (kernels/fa_forward.hip:258); keep iff (r0>>8)/2^24 >= p, kept
 * values scaled by 1/(1-p); the row sum is taken before dropout.
 * -------------------------------------------------------------------------------------------*/
typedef struct FaFwdParams {
  unsigned int struct_size;
  const void* Q; const void* K; const void* V;
  void* O;
  float* LSE;                          /* optional */
  FaStrides sQ, sK, sV, sO;
  int batch;
  int SQ, SK, HD, NH, gqa;             /* gqa = NH / (number of kv heads) */
  float scale, softcap;                /* softcap <= 0 disables */
  int causal, win_left, win_right;     /* window bounds < 0 = unbounded */
  int attn_chunk;                      /* 0 disables */
  const float* alibi_slopes;           /* [NH] or null */
  float dropout_p;
  unsigned long long philox_seed;
  const int* cu_q; const int* cu_k;    /* varlen: [batch+1] int32, or null */
  const int* seqused_q; const int* seqused_k;   /* varlen: [batch] int32, or null */
  long long lse_total_q;               /* varlen LSE row length (total tokens of q) */
  const unsigned int* dropout_bits;    /* optional precomputed keep mask (fa_dropout_mask_launch,
                                          dense only); null = Philox evaluated in the kernel */
  long long total_k;                   /* varlen: rows of K and V (total key tokens).  The tensor-core
                                          kernel needs it (with lse_total_q as the rows of Q and O) to
                                          bound its TMA boxes; 0 = unknown, the CUDA-core kernel runs */
  /* paged K/V (varlen only; flash_attn_varlen_func's block_table): K and V are caches
   * [num_blocks, page, NH/gqa, HD] contiguous, key position k of sequence z sits in page
   * block_table[z * max_blocks + k / page], slot k % page; cu_k (or seqused_k) gives the key
   * counts and sK / sV are ignored.  An entry outside [0, num_blocks) reads page 0 and raises
   * fa_device_error bit 1024.  Replaces the reference's page unrolling before the forward
   * (package/fable_attn/flash_attn_interface.py:438-472).  block_table null = not paged. */
  const int* block_table;
  int page, max_blocks;
  long long num_blocks;
  /* Optional rotary embedding of Q inside the kernel (rot_cos null = none): each Q row is rotated
   * as it lands in shared memory, with the roundings of fa_rotary_launch (the reference's torch
   * arithmetic, layers/rotary.py:20-68); position = the row's index in its sequence, rot_cos /
   * rot_sin fp32 [rot_seqlen_ro, rot_dim / 2], NeoX pairs (j, j + rot_dim/2) or interleaved
   * (2j, 2j + 1).  K is not rotated here: rotate it once beforehand (fa_rotary_launch); it is read
   * by many CTAs.  fp16/bf16 only (FA_ERR_UNSUPPORTED otherwise).  A
   * position past the table leaves its row unrotated and raises fa_device_error bit 4096. */
  const float* rot_cos;
  const float* rot_sin;
  int rot_dim, rot_seqlen_ro, rot_interleaved;
} FaFwdParams;

FA_API int fa_forward_launch(const FaFwdParams* p, int dtype, void* stream);

/* ------------------------------------------------------------------------------------------
 * Backward.  Replaces BwdParams / fable_attn_backward_launch.  Computes dQ, dK, dV with no
 * atomics (bit-reproducible): a preprocessing kernel writes dsum = rowsum(O*dO), a dK/dV kernel
 * per key tile sums over every query tile and every query head of the kv group, and a dQ kernel
 * per query tile sums over key tiles (kernels/backward.hip:86-387).  dsum is caller-provided
 * workspace of [B, Hq, SQ] fp32 (varlen: [Hq, lse_total_q]).  Dense or varlen (cu_q/cu_k),
 * same geometry rules as the forward.  The mask is the forward's without attn_chunk
 * (kernels/backward.hip:76-83); dropout recomputes the forward's Philox mask bit-identically.
 * -------------------------------------------------------------------------------------------*/
typedef struct FaBwdParams {
  unsigned int struct_size;
  const void *Q, *K, *V, *O, *dO;
  void *dQ, *dK, *dV;
  const float* lse;                    /* forward LSE, same layout as FaFwdParams.LSE */
  float* dsum;                         /* workspace, same layout as lse */
  FaStrides qs, ks, vs, os, dos, dqs, dks, dvs;
  int B, Hq, Hk, SQ, SK, D, gqa;
  float scale, softcap;
  const float* alibi;
  int causal, win_left, win_right;
  int dropout;
  unsigned long long drop_seed;
  float dropout_p, keep_scale;
  const int* cu_q; const int* cu_k;
  const int* seqused_q; const int* seqused_k;
  long long lse_total_q;
  const unsigned int* dropout_bits;    /* optional precomputed keep mask, as in FaFwdParams */
  long long total_k;                   /* varlen: rows of K and V, as in FaFwdParams */
  /* optional workspace of fa_dropout_mask_words(Hq, SK, SQ) words (dense, with dropout_bits): the
   * backward writes the key-major copy of dropout_bits there, layout [Hq][ceil(SQ/32)][SK] with bit
   * r of word (h, qw, k) = keep decision of (query row 32 qw + r, key k), and its dK/dV kernel reads
   * it instead of transposing the row-major words itself.  NULL: the transpose stays in the kernel. */
  unsigned int* dropout_bits_t;
} FaBwdParams;

FA_API int fable_attn_backward_launch(const FaBwdParams* p, int dtype, void* stream);

/* ------------------------------------------------------------------------------------------
 * Dropout keep mask as bits, computed once and read by the forward and backward kernels in place
 * of evaluating Philox per score.  No counterpart in the reference (its kernels evaluate Philox
 * per score, kernels/fa_forward.hip:255-259, kernels/backward.hip:171-173); the bits are exactly
 * the reference's keep decisions: bit k%32 of word bits[(h*W + k/32)*SQ + q], W = ceil(SK/32),
 * is 1 iff Philox(seed, (h*SQ + q)*SK + k) keeps (q, k) with drop probability p.  Words are
 * query-row-minor so that 32 consecutive rows read one 128-byte line.  The mask has no batch
 * term, like the reference's.  Only words holding a key that row q can see under (causal,
 * win_left, win_right) are written; consumers read no others.  Dense layouts only.
 * -------------------------------------------------------------------------------------------*/
FA_API long long fa_dropout_mask_words(int NH, int SQ, int SK);
FA_API int fa_dropout_mask_launch(unsigned long long seed, float p, int NH, int SQ, int SK, int causal, int win_left,
                                  int win_right, unsigned int* bits, void* stream);

/* ------------------------------------------------------------------------------------------
 * Rotary position embedding of q or k, one HBM pass.  Replaces the torch arithmetic of
 * apply_rotary_emb (package/fable_attn/layers/rotary.py:20-68) for device tensors, with the same
 * roundings (cos/sin cast to x's dtype, each product and sum rounded to it), so the result is
 * bit-identical to the reference's.  x / out are [rows][heads][dim] with element strides
 * (dim contiguous); out == x rotates in place, otherwise dims past rotary_dim are copied.
 *   dense:  rows = batch * seqlen, row b*seqlen + s sits at position s + offset(b)
 *   varlen: cu_seqlens [batch+1] int32, row t of sequence i sits at t - cu[i] + offset(i)
 * offset(b) = offsets ? offsets[b] : offset.  cos/sin [seqlen_ro][rotary_dim/2] fp32.
 * interleaved: pairs (2j, 2j+1) (GPT-J); else (j, j + rotary_dim/2) (NeoX).  A position outside
 * the table leaves its row unrotated and raises fa_device_error bit 256.  No counterpart in
 * the reference's C++ (its rotary is torch code).
 * -------------------------------------------------------------------------------------------*/
typedef struct FaRotaryParams {
  unsigned int struct_size;
  const void* x;
  void* out;
  long long rows;
  int heads, dim, rotary_dim;
  long long x_row_stride, x_head_stride, out_row_stride, out_head_stride;
  int seqlen;                          /* dense rows per sequence */
  const int* cu_seqlens;               /* varlen [batch+1] or null */
  int batch;
  int offset;                          /* position offset for every sequence ... */
  const int* offsets;                  /* ... or per sequence [batch] */
  const float* cos; const float* sin;
  int seqlen_ro;                       /* rows of the cos / sin tables */
  int interleaved;
} FaRotaryParams;

FA_API int fa_rotary_launch(const FaRotaryParams* p, int dtype, void* stream);

/* ------------------------------------------------------------------------------------------
 * Paged-KV decode (one or several new tokens per sequence).  Replaces DecParams /
 * fa_decode_launch (kernels/fa_decode.hip:343-362).
 *   q         [batch, nq, NH, HD] contiguous (nq new tokens per sequence)
 *   Kc, Vc    paged cache [num_blocks, page, NH/gqa, HD] contiguous; page a power of two
 *   block_table [batch, max_blocks] int32 (row stride max_blocks)
 *   ctx_len   [batch] int32: cache length BEFORE this call's append (flash-attn cache_seqlens)
 *   o         [batch, nq, NH, HD]
 *   scratch   fp32 workspace of fa_decode_scratch_floats(...) floats (split-K partials)
 *   lse_out   optional [batch, nq, NH] fp32, natural log
 * New token tk sits at position ctx_len+tk; it sees keys [lo, ctx_len) plus, when new_k/new_v
 * are given (appended at ctx_len.. before attention, rotary applied to k), the new keys up to
 * and including its own.  lo = max(leftpad, pos - window + 1) (window < 0 = unbounded).
 * Rotary (1 = NeoX halves, 2 = interleaved pairs) rotates q (and appended k) by the table row
 * cos/sin[rotary_pos ? rotary_pos[b]+tk : ctx_len[b]+tk], rotary_dim dims (0 = all).
 * softcap/alibi as in the forward with query position ctx_len+tk.  Any gqa is supported
 * (the reference's kernel covers only gqa in {1,2,4,8}, kernels/fa_decode.hip:326-331).
 * nsplit: number of KV splits per sequence (fa_decode_num_splits gives the default).
 * -------------------------------------------------------------------------------------------*/
typedef struct FaDecParams {
  unsigned int struct_size;
  const void* q;
  void* Kc; void* Vc;
  const int* block_table;
  void* o;
  float* scratch;
  const int* ctx_len;
  const float* cos; const float* sin;
  int batch, NH, gqa, HD, page, max_blocks, nsplit, window;
  int rotary;                          /* 0 none, 1 neox, 2 interleaved */
  float scale;
  const int* leftpad;                  /* [batch] or null */
  float* lse_out;                      /* [batch, nq, NH] or null */
  float softcap;
  const float* alibi;                  /* [NH] or null */
  int nq;
  int append;                          /* set by fa_decode_launch: new_k/new_v given */
  int rotary_dim;                      /* 0 = HD */
  const int* rotary_pos;               /* [batch] or null */
  long long num_blocks;                /* pages in the cache (block_table entries are checked
                                          against it on the device; out-of-range pages read as
                                          empty and set the error flag) */
  int* err_flag;                       /* optional device int set non-zero on a bad page index */
  int o_f32;                           /* 1: o is fp32 (for callers that merge partial results further,
                                          e.g. a KV range split across GPUs); 0: o has q's dtype */
} FaDecParams;

FA_API int fa_decode_launch(const FaDecParams* p, int dtype, void* stream,
                     const void* new_k, const void* new_v);

/* ------------------------------------------------------------------------------------------
 * fa_decode_launch_noalloc — the same decode, for callers that cannot allocate device memory at
 * call time.  No counterpart in the reference: its decode always allocates its split-K scratch
 * through torch (package/csrc/dispatch.cpp:203).
 *
 * Who needs it: hosts that bind only this C ABI from another runtime (a Go, Java or Rust serving
 * process with no CUDA allocator of its own), processes whose device memory is reserved up front
 * by a pool (a KV-cache manager or caching allocator holding most of HBM, where one more
 * cudaMalloc can fail), and decode loops that cannot afford cudaMalloc/cudaFree in the step
 * (cudaFree synchronises the device).  The caller still passes every input and output; only the
 * split-K scratch is taken from a fixed device array of FA_DECODE_NOALLOC_MAX_SCRATCH_FLOATS
 * floats (16 MiB) inside the library, which every GPU that loads the library holds until exit.
 *   - p->scratch is ignored (may be null).  Requests needing more scratch than the array holds
 *     (fa_decode_scratch_floats(batch, nq, NH, HD, nsplit) > the maximum) are refused with
 *     FA_ERR_SIZE before any work; lower nsplit to fit.
 *   - Each call looks up the array's device address on the current device
 *     (cudaGetSymbolAddress); the first call on a device also loads the library's kernels there,
 *     so make that first call before any stream capture.
 *   - No allocation of any kind: no cudaMalloc/cudaFree, no library allocator.
 *   - All calls share the one array and it keeps the last call's contents.  Nothing in it needs
 *     to start at zero (every split writes its whole slot before the merge reads it), but calls
 *     whose kernels overlap on the GPU (different streams, or several host threads) race on it:
 *     serialise them on one stream.
 * -------------------------------------------------------------------------------------------*/
#define FA_DECODE_NOALLOC_MAX_SCRATCH_FLOATS (4LL << 20)
FA_API int fa_decode_launch_noalloc(const FaDecParams* p, int dtype, void* stream, const void* new_k,
                                    const void* new_v);

/* Default split count: enough CTAs to fill the GPU, each split at least 256 positions, at most
 * 512 splits; num_splits > 0 is taken as given (clamped to [1, 512]). */
FA_API int fa_decode_num_splits(int batch, int nq, int nheads_kv, long long ctx_bound, int num_splits);

/* Floats of scratch fa_decode_launch needs for these sizes. */
FA_API long long fa_decode_scratch_floats(int batch, int nq, int NH, int HD, int nsplit);

/* ------------------------------------------------------------------------------------------
 * LSE-merge of split-KV partial results (flash_attn_combine).
 *   out_partial [nsplit, B, S, H, D] (dtype in_dtype), lse_partial [nsplit, B, H, S] fp32,
 *   out [B, S, H, D] (dtype out_dtype), lse_out optional [B, H, S] fp32; all contiguous.
 *   out = sum_s w_s*out_s / sum_s w_s with w_s = exp(lse_s - max_s lse_s); a row whose
 *   partials are all -inf gives 0.
 * -------------------------------------------------------------------------------------------*/
typedef struct FaCombineParams {
  unsigned int struct_size;
  const void* out_partial; int in_dtype;
  const float* lse_partial;
  void* out; int out_dtype;
  float* lse_out;
  int nsplit, B, S, H, D;
  /* Packed partials, e.g. the buffer one all-gather of every rank's (out, lse) produces (0 = the
   * contiguous layouts above): out_split_stride = elements from one split's partial output to the
   * next, lse_split_stride = floats from one split's LSE to the next, lse_bsh = 1 when each split's
   * LSE rows are ordered (b, s, h) like the output rows instead of (b, h, s). */
  long long out_split_stride, lse_split_stride;
  int lse_bsh;
} FaCombineParams;

FA_API int fa_combine_launch(const FaCombineParams* p, void* stream);

/* ------------------------------------------------------------------------------------------
 * Multi-GPU decode exchange over peer memory (no counterpart in the reference, which has no
 * multi-GPU layer; its merge rule is flash_attn_combine, package/fable_attn/flash_attn_interface.py
 * :567-580).  A decode whose KV range is split across `world` GPUs leaves on every rank a packed
 * partial: rows = B*S*H output rows of D fp32 values, then the rows' fp32 LSE, rows in (b, s, h)
 * order (fa_decode_launch with o_f32 and lse_out pointing into the buffer).  All ranks' buffers
 * live in one symmetric allocation, so every rank reaches every other rank's through a peer
 * pointer (NVLink P2P loads; no multicast, no library kernel on peer memory).
 *   fa_peer_merge_launch    : publishes "ready" for the current step to every peer, waits (bounded)
 *                             until every peer is ready, then merges each row from all ranks'
 *                             buffers into out [B, S, H, D] (out_dtype) and optionally lse_out
 *                             [B, H, S].
 *   fa_peer_step_end_launch : publishes "done", waits (bounded) until every peer is done (the
 *                             buffers may then be overwritten by the next step), advances *step.
 * Two ways to run it, every rank running the same steps on one stream:
 *   one slot  (slot_floats = 0): per step the decode into the own buffer, the merge, the step end;
 *   two slots (slot_floats = the floats of one packed partial, each buffer holding two): step s
 *             (counted from 1) uses slot (s - 1) % 2; per step the decode into that slot and the
 *             merge, which then also advances *step (its last CTA).  A slot is rewritten two steps
 *             later, after every peer has published "ready" for the step in between (which it does
 *             only once its previous merge has finished reading), so no step end is needed.
 * The step number lives on the device (*step, start at 0; done_ctas, a device int starting at 0,
 * counts the merge's finished CTAs in two-slot mode), so captured CUDA graphs replay correctly
 * (in two-slot mode a graph holds an even number of steps, the host picking the slot).
 * peer_signals[r] points at rank r's signal words (at least 2 * world uint32, zero before the first
 * step): word r' of rank r holds rank r''s ready step, word world + r' its done step.  A wait that
 * exceeds wait_ns (0 = 2 s) sets FA_PEER_ERR_WAIT in *err_flag (when given) and the kernel carries
 * on without hanging.
 * -------------------------------------------------------------------------------------------*/
#define FA_PEER_MAX_WORLD 8
#define FA_PEER_ERR_WAIT 1
typedef struct FaPeerMergeParams {
  unsigned int struct_size;
  const float* const* peer_bufs;       /* device array [world]: each rank's packed partial */
  unsigned int* const* peer_signals;   /* device array [world]: each rank's signal words */
  int rank, world;
  int B, S, H, D;                      /* D a multiple of 4 */
  void* out; int out_dtype;
  float* lse_out;                      /* optional [B, H, S] */
  int* step;                           /* this rank's device step counter */
  int* err_flag;                       /* optional device int */
  unsigned long long wait_ns;          /* bound of each wait; 0 = 2 s */
  long long slot_floats;               /* two-slot mode: floats per slot; 0 = one slot */
  int* done_ctas;                      /* two-slot mode: device int, 0 before the first step */
} FaPeerMergeParams;

FA_API int fa_peer_merge_launch(const FaPeerMergeParams* p, void* stream);
FA_API int fa_peer_step_end_launch(const FaPeerMergeParams* p, void* stream);

/* ---- introspection ---- */
FA_API int fa_abi_version(void);
FA_API const char* fa_last_error(void);       /* message of the last failing call on this thread */
/* Error bits recorded on the device (0 = none).  A bounded wait in a tensor-core kernel that
 * times out records a bit here and the kernel unwinds instead of hanging (its outputs are then
 * not valid); bits 1024 / 4096 / 256 flag a paged-K/V entry outside the cache and a rotary
 * position outside the cos/sin table.  Synchronous (device -> host copy); clear != 0 resets the
 * bits.  No counterpart in the reference (its kernels have no waits that can give up). */
FA_API int fa_device_error(int clear);
/* Bit of fa_device_error set by fa_wait_selftest. */
#define FA_DEVERR_WAIT_SELFTEST 65536
/* Launches one tiny kernel whose bounded wait can never be satisfied (nothing arrives on its
 * mbarrier and nothing is in flight): after limit_ns (0 < limit_ns <= 1e10) the wait gives up,
 * records FA_DEVERR_WAIT_SELFTEST in fa_device_error and the kernel returns.  Lets a host check
 * the give-up path of the pipelines' waits without faulting or hanging a GPU.  No counterpart in
 * the reference. */
FA_API int fa_wait_selftest(unsigned long long limit_ns, void* stream);
/* Number of this library's kernels launched since load (all threads, all devices). */
FA_API unsigned long long fa_kernel_launch_count(void);
/* 1 when the forward's two-query-tile kernel (dense fp16/bf16, head_dim 128, no softcap / alibi /
 * dropout) can run on the current device with this build, 0 otherwise (those requests then run on
 * the one-tile kernel).  Needs a device; makes no launch. */
FA_API int fa_forward_two_tile_ready(int bf16);

#ifdef __cplusplus
}
#endif
#endif /* FABLE_ATTN_H */
