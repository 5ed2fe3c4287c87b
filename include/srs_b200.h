/*
 * srs_b200.h — C ABI of the sm_100a stochastic-rounding optimizer library.
 *
 * Every entry point takes plain device addresses, element counts, POD
 * scalars and a cudaStream_t passed as `void*`.  Nothing here allocates
 * device memory: callers own every buffer (inputs, outputs and the row
 * tables of the multi-tensor steps).  Work is enqueued on the given stream
 * of the calling thread's current device; no entry point synchronises.
 *
 * Return value: SRS_OK (0) or a negative SRS_ERR_* code.  The text of the
 * most recent failure on the calling thread is available from
 * srs_last_error().  No entry point aborts the process.
 *
 * Counter-hash RNG contract (identical to the Python `sr_states` package):
 *   h32(x)        x ^= x>>16; x *= 0x7FEB352D; x ^= x>>15; x *= 0x846CA68B; x ^= x>>16   (mod 2^32)
 *   update_key    k = h32(seed_lo ^ 0x9E3779B9); k = h32(k ^ seed_hi); k = h32(k ^ step_lo);
 *                 k = h32(k ^ step_hi); k = h32(k ^ param_index)
 *   state_key     h32(update_key ^ state_index)
 *   element e of a stored state uses h32((e + offset + state_key) mod 2^32);
 *   element e of a standalone cast uses h32((e + offset + seed) mod 2^32).
 */
#ifndef SRS_B200_H
#define SRS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SRS_ABI_VERSION 6

/* ---- status codes ------------------------------------------------------ */
#define SRS_OK 0
#define SRS_ERR_INVALID_ARGUMENT (-1) /* bad pointer, size, format, rule or flag */
#define SRS_ERR_UNSUPPORTED_DEVICE (-2) /* current device is not compute capability 10.0 */
#define SRS_ERR_CUDA (-3)             /* a CUDA runtime call failed (launch, attribute query) */

/* ---- storage formats (state, cast output) ------------------------------ */
#define SRS_FMT_F32 0
#define SRS_FMT_BF16 1
#define SRS_FMT_F16 2
#define SRS_FMT_E4M3 3 /* torch.float8_e4m3fn, saturating to +-448 */
#define SRS_FMT_E5M2 4 /* torch.float8_e5m2, saturating to +-57344 */

/* ---- rounding rules ---------------------------------------------------- */
#define SRS_RULE_NEAREST 0    /* round to nearest, ties to even */
#define SRS_RULE_STOCHASTIC 1 /* counter-hash stochastic rounding */
/* Round toward zero: the format's value of largest magnitude not above |x|,
 * sign kept (BF16: the high half of the FP32 encoding).  Finite values never
 * become infinite; +-Inf stays infinite in BF16/FP16 and saturates in FP8; NaN
 * is stored as under the other rules.  Not a reference built-in: it is the
 * native implementation a custom rule registered through
 * register_rounding(..., native="toward_zero") runs (the reference's custom
 * rules, sr_states/rounding.py:28-66, run as Triton callbacks). */
#define SRS_RULE_TOWARD_ZERO 2

/* ---- multi-tensor row table -------------------------------------------- */
#define SRS_ROW_PARAM_BF16 0x1u  /* parameter is BF16 (else FP32) */
#define SRS_ROW_GRAD_BF16 0x2u   /* gradient is BF16 (else FP32) */
#define SRS_ROW_VECTOR_OK 0x4u   /* every base address is aligned for 8-element vector access */
#define SRS_ROW_CLASS_SHIFT 8    /* bits 8..15: index of the row's AdamW step class */
#define SRS_MAX_STEP_CLASSES 32
/* `uniform_kind` of the multi-tensor steps: the (SRS_ROW_PARAM_BF16 |
 * SRS_ROW_GRAD_BF16) bits every row shares, or SRS_KIND_MIXED.  It selects a
 * kernel specialised for that dtype pair; rows that do not match it still run
 * correctly on a generic path. */
#define SRS_KIND_MIXED 0xFFFFFFFFu

/*
 * One row = one contiguous run of `numel` elements of one parameter (a whole
 * parameter, or its intersection with this rank's ZeRO-1 shard).  Rows are
 * ordered by tile_begin; row i covers tiles [tile_begin_i, tile_begin_{i+1})
 * and tile_begin_i + ceil(numel_i / srs_tile_elems()) == tile_begin_{i+1}.
 */
typedef struct srs_row {
  uint64_t param;       /* device address of the parameter run (FP32 or BF16)    */
  uint64_t grad;        /* device address of the gradient run (FP32 or BF16)     */
  uint64_t state[2];    /* device addresses of the state runs (state[1]: AdamW)  */
  int64_t numel;        /* > 0                                                    */
  int64_t tile_begin;   /* first tile of this row in the launch's tile space      */
  uint32_t param_index; /* global parameter position (low 32 bits), or the update
                           key itself when the launch uses SRS_KEY_GIVEN          */
  uint32_t offset;      /* flat element index of element 0 within its parameter,
                           mod 2^32 (the shard start of the RNG contract)        */
  uint32_t flags;       /* SRS_ROW_* bits and the step class                     */
  uint32_t reserved;    /* zero                                                   */
} srs_row;

/* How the per-row update key is obtained. */
#define SRS_KEY_DERIVE 0 /* update_key(seed words, step words, row.param_index) */
#define SRS_KEY_GIVEN 1  /* row.param_index already holds the update key        */

typedef struct srs_rng {
  uint32_t seed_lo, seed_hi; /* low 64 bits of the group seed   */
  uint32_t step_lo, step_hi; /* low 64 bits of the global RNG step */
  int32_t key_mode;          /* SRS_KEY_DERIVE or SRS_KEY_GIVEN  */
} srs_rng;

/*
 * AdamW scalars, each the FP32 rounding of the double-precision expression:
 *   beta1, beta2, one_minus_beta1 = 1-beta1, one_minus_beta2 = 1-beta2,
 *   eps, decay = 1 - lr*weight_decay,
 *   per step class c (bias-correction step t_c):
 *     neg_step_size[c] = -lr / (1 - beta1^t_c),  bias2_sqrt[c] = (1 - beta2^t_c)^0.5
 * Per element (FP32, each operation rounded once):
 *   m' = fma(g, 1-b1, m*b1);  v' = fma((1-b2)*g, g, v*b2)
 *   d  = sqrt(v') / bias2_sqrt + eps;  p' = p*decay + (neg_step_size*m') / d
 */
typedef struct srs_adamw_hparams {
  float beta1, beta2, one_minus_beta1, one_minus_beta2;
  float eps, decay;
  int32_t n_step_classes; /* 1..SRS_MAX_STEP_CLASSES */
  float neg_step_size[SRS_MAX_STEP_CLASSES];
  float bias2_sqrt[SRS_MAX_STEP_CLASSES];
} srs_adamw_hparams;

/* SGDM scalars: u' = u*momentum + g;  p' = fma(u', neg_lr, p), neg_lr = -lr. */
typedef struct srs_sgdm_hparams {
  float momentum;
  float neg_lr;
} srs_sgdm_hparams;

/* ---- library information ----------------------------------------------- */
int srs_abi_version(void);
/* Elements per tile of the multi-tensor steps (row tile_begin arithmetic). */
int64_t srs_tile_elems(void);
/* Text of the last failure on this thread ("" if none). */
const char* srs_last_error(void);
/* SRS_OK if the current device can run the kernels (compute capability 10.0). */
int srs_check_device(void);

/* ---- standalone cast ---------------------------------------------------
 * Replaces sr_states/triton/cast.py:32-60 (`cast`) and
 * sr_states/triton/sr_cast.py:89-128 (`sr_cast_bf16`, `rn_cast_bf16`).
 * y[e] = round(x[e]) into `out_format` under `rule`; the stochastic counter of
 * element e is (e + offset + seed) mod 2^32.  SRS_FMT_F32 copies.  x and y must
 * not overlap.  n == 0 is a no-op.
 */
int srs_cast(const float* x, void* y, int64_t n, int out_format, int rule, uint32_t seed,
             uint32_t offset, int grid_ctas, void* stream);

/* ---- fused multi-tensor steps -------------------------------------------
 * Replace the per-bucket launches of sr_states/triton/adamw.py:303-317
 * (_multi_adamw_kernel) and sr_states/triton/sgd.py:214-237
 * (_multi_sgdm_kernel): ONE launch covers every row of a parameter group on
 * one device, whatever the rows' parameter/gradient dtypes and AdamW
 * bias-correction steps.  `rows` is a device array of n_rows srs_row;
 * n_tiles = tile_begin of the last row + its tile count.  grid_ctas <= 0
 * selects the persistent grid (a multiple of the SM count).
 */
int srs_adamw_multi(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int m_format,
                    int m_rule, int v_format, int v_rule, const srs_adamw_hparams* hp,
                    const srs_rng* rng, uint32_t uniform_kind, int grid_ctas, void* stream);

int srs_sgdm_multi(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int u_format,
                   int u_rule, const srs_sgdm_hparams* hp, const srs_rng* rng,
                   uint32_t uniform_kind, int grid_ctas, void* stream);

/* ---- fused step + all-gather over peer memory ----------------------------
 * No counterpart in the reference (it has no sharded step; this is the
 * ZeRO-1 all-gather of the updated parameters fused into the step).  With
 * every rank's parameters in a flat buffer of identical layout, the step
 * stores each updated parameter vector both locally and at the same offset of
 * every peer's buffer (plain stores through NVLink peer mappings), so no
 * separate all-gather runs.  delta_*[w] = (peer w's buffer) - (this rank's
 * buffer) in this process's address space, for FP32 and BF16 parameters.
 * The caller orders the step against the peers (a barrier before, so no peer
 * still reads its replica, and one after, before anyone uses the result).
 */
#define SRS_MAX_PEERS 7
/* How the updated parameters reach the replicas (srs_peers.mode):
 *   SRS_PEERS_STORE      each vector is stored locally and at delta_*[w] for
 *                        every peer w (plain stores through peer mappings);
 *   SRS_PEERS_MULTICAST  the caller's flat buffers are bound to an NVLink
 *                        multicast object spanning every rank (this one
 *                        included) and mc_delta_* = (multicast address of the
 *                        buffer) - (this rank's buffer): each aligned 8-element
 *                        vector is written ONCE, with multimem.st, and NVSwitch
 *                        delivers it to every replica, the local one included.
 *                        Elements outside aligned vectors (row tails, rows
 *                        without SRS_ROW_VECTOR_OK), which multimem cannot
 *                        store at 2-byte granularity, take the SRS_PEERS_STORE
 *                        path, so delta_*[] must hold the peers as well.
 * Both end with a system-scope fence (and a proxy fence for the multicast
 * alias), so the caller's barrier after the step publishes every replica. */
#define SRS_PEERS_STORE 0
#define SRS_PEERS_MULTICAST 1
typedef struct srs_peers {
  int32_t n_peers; /* 0..SRS_MAX_PEERS */
  int32_t mode;    /* SRS_PEERS_STORE or SRS_PEERS_MULTICAST */
  int64_t delta_f32[SRS_MAX_PEERS];
  int64_t delta_bf16[SRS_MAX_PEERS];
  int64_t mc_delta_f32;  /* SRS_PEERS_MULTICAST: multicast address - local buffer */
  int64_t mc_delta_bf16;
} srs_peers;

int srs_adamw_multi_gather(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int m_format,
                           int m_rule, int v_format, int v_rule, const srs_adamw_hparams* hp,
                           const srs_rng* rng, uint32_t uniform_kind, const srs_peers* peers,
                           int grid_ctas, void* stream);

int srs_sgdm_multi_gather(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int u_format,
                          int u_rule, const srs_sgdm_hparams* hp, const srs_rng* rng,
                          uint32_t uniform_kind, const srs_peers* peers, int grid_ctas,
                          void* stream);

/* ---- tile ranges and copies for a pipelined exchange ---------------------
 * No counterpart in the reference.  The same steps over the tiles
 * [tile_lo, tile_hi) of the table only (0 <= tile_lo <= tile_hi <= n_tiles):
 * a sharded step split into chunks, each chunk's updated parameters sent to
 * the peers by srs_copy_async (a device-to-device cudaMemcpyAsync, done by
 * the copy engines) while the next chunk is updated.  `peers` (may be NULL)
 * are replicas the range's kernel stores to itself, as in the *_gather entry
 * points, so some peers can be served by the kernel and others by the copy
 * engines.
 */
int srs_adamw_multi_range(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int64_t tile_lo,
                          int64_t tile_hi, int m_format, int m_rule, int v_format, int v_rule,
                          const srs_adamw_hparams* hp, const srs_rng* rng, uint32_t uniform_kind,
                          const srs_peers* peers, int grid_ctas, void* stream);

int srs_sgdm_multi_range(const srs_row* rows, int64_t n_rows, int64_t n_tiles, int64_t tile_lo,
                         int64_t tile_hi, int u_format, int u_rule, const srs_sgdm_hparams* hp,
                         const srs_rng* rng, uint32_t uniform_kind, const srs_peers* peers,
                         int grid_ctas, void* stream);

int srs_copy_async(void* dst, const void* src, uint64_t bytes, void* stream);

/* Peer mappings (CUDA IPC) of the buffers above.  srs_ipc_export writes a
 * handle of the allocation holding device address `p` (SRS_IPC_HANDLE_BYTES
 * bytes) and the offset of `p` inside it; srs_ipc_import maps a peer's
 * allocation into this process on the current device; srs_ipc_close unmaps
 * it.  Allocations from the virtual-memory API (expandable segments) cannot
 * be exported: srs_ipc_export then fails and the caller keeps a collective. */
#define SRS_IPC_HANDLE_BYTES 64
int srs_ipc_export(const void* p, void* handle, uint64_t* offset);
int srs_ipc_import(const void* handle, void** base);
int srs_ipc_close(void* base);

/* ---- multi-tensor AdamW step that allocates nothing ----------------------
 * No counterpart in the reference.  Same update as srs_adamw_multi, for
 * callers that cannot allocate device memory at step time (a runtime whose
 * allocator is reserved or already full, or a step issued from code that must
 * not call into any allocator).  `host_rows` is a HOST array of n_rows srs_row,
 * copied on `stream` into a fixed device-resident table of
 * SRS_NOALLOC_MAX_ROWS rows that every call on a device shares.  The copy is an
 * ordinary host-to-device cudaMemcpyAsync on `stream`: keep host_rows valid and
 * unchanged until the step has run on the stream.  The parameter/gradient
 * dtype kind is read from the rows.
 * Limits and rules:
 *   - n_rows > SRS_NOALLOC_MAX_ROWS fails with SRS_ERR_INVALID_ARGUMENT;
 *   - rows are checked on the host before anything is enqueued: tile_begin
 *     prefix sums, n_tiles, step classes, null addresses, and the alignment a
 *     row's SRS_ROW_VECTOR_OK flag promises (16 bytes for parameters,
 *     gradients and 2- or 4-byte states, 8 bytes for FP8 states); a violation
 *     fails with SRS_ERR_INVALID_ARGUMENT;
 *   - the first call on a device looks up the table's address (set-up); make
 *     that first call before any stream capture (a first call made during
 *     capture fails with SRS_ERR_INVALID_ARGUMENT);
 *   - a call captured into a CUDA graph captures the row copy too, which then
 *     reads host_rows at every replay: under capture host_rows must be
 *     page-locked (cudaHostAlloc / cudaHostRegister; pageable rows fail with
 *     SRS_ERR_INVALID_ARGUMENT) and stay valid while the graph can be
 *     replayed; a replay uses the rows' contents at that time, but the
 *     hyperparameters and RNG words captured with the call;
 *   - calls on one device that can overlap in time (different streams or host
 *     threads without ordering) race on the shared table: order them.
 */
#define SRS_NOALLOC_MAX_ROWS 4096
int srs_adamw_multi_noalloc(const srs_row* host_rows, int64_t n_rows, int64_t n_tiles,
                            int m_format, int m_rule, int v_format, int v_rule,
                            const srs_adamw_hparams* hp, const srs_rng* rng, int grid_ctas,
                            void* stream);

/* ---- fused single-tensor steps ------------------------------------------
 * Replace sr_states/triton/adamw.py:160-221 (`triton_adamw_step_`) and
 * sr_states/triton/sgd.py:115-171 (`triton_sgdm_step_`).  `row` is a HOST
 * srs_row describing one tensor; its param_index field holds the update key
 * (the functional API's `seed`).  hp->n_step_classes must be 1.
 */
int srs_adamw_single(const srs_row* row, int m_format, int m_rule, int v_format, int v_rule,
                     const srs_adamw_hparams* hp, int grid_ctas, void* stream);

int srs_sgdm_single(const srs_row* row, int u_format, int u_rule, const srs_sgdm_hparams* hp,
                    int grid_ctas, void* stream);

/* ---- RNG key derivation on the device ----------------------------------
 * Mirrors sr_states/triton/_keys.py:20-30 (_update_key/_state_key), used to
 * check that device keys equal host keys.  For each i < n writes
 * out[3i..3i+2] = {update_key(words, param_index[i]), state_key(k, 0), state_key(k, 1)}.
 */
int srs_derive_keys(const uint32_t* param_index, uint32_t* out, int64_t n, const srs_rng* rng,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SRS_B200_H */
