/*
 * kvb.h - C ABI of the B200 (sm_100a) packed-KV decode path.
 *
 * Drop-in native replacement for the decode-time hot path of TahirSher/KV-Project's KV-cache
 * compression methods (STRATA_KV.py, QUASAR_KV.py, HEDGE_KV.py, TILT_KV.py, LCTC_KV.py, KV_LDT).
 * Every entry point takes plain device pointers, 64-bit sizes and a cudaStream_t passed as void*.
 * No call allocates device memory or synchronises the stream, except kvb_device_status (which
 * reads the device status word).  Errors come back as a kvb_status; kvb_last_error() returns a
 * thread-local description of the last failure.
 *
 * Numerics contract (checked by tests/ against the reference on identical seeded inputs):
 *   - codes, fp16 scales / zero points and selected index sets are bit-exact;
 *   - attention outputs agree with the reference's float32 dequantise-then-attend result
 *     (chunked_attention, STRATA_KV.py:641) within max-abs 2e-3.
 */
#ifndef KVB_H
#define KVB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int kvb_status;
#define KVB_OK 0
#define KVB_EINVAL 1          /* bad shape, dtype, stride, alignment or size */
#define KVB_ECUDA 2           /* a CUDA runtime call failed (message in kvb_last_error) */
#define KVB_ETIMEDOUT 3       /* a bounded device wait gave up (device status word set) */
#define KVB_EUNSUPPORTED 4    /* valid request outside the instantiated kernel set */

/* element types */
#define KVB_F32 0
#define KVB_F16 1
#define KVB_BF16 2
#define KVB_F64 3

/* how a stored vector is coded */
#define KVB_CODE_ASYM 0       /* KIVI: per group fp16 (lo, scale) pair, x ~ code * scale + lo */
#define KVB_CODE_MIDRISE 1    /* STRATA: one fp16 scale s per vector, x ~ (code - (2^b - 1) / 2) * s */

/* grouping of the key code (values are always grouped per token) */
#define KVB_K_PER_TOKEN 0     /* groups of `group` channels inside each token (or one scale per token) */
#define KVB_K_PER_CHANNEL 1   /* per channel over groups of `group` consecutive stored tokens */

const char* kvb_last_error(void);
int kvb_version(void);

/* Device status word (bit 0: a bounded wait timed out; bit 1: a bounds check failed; bit 2: a NaN
 * key reached kvb_rank_split, whose ranking is then undefined; bit 3: a decode workspace was not
 * zero-filled before its first use, so that call's merge may be wrong).  Synchronises
 * `stream`, copies the word to *out and clears it when `clear` is non-zero. */
kvb_status kvb_device_status(unsigned* out, int clear, void* stream);

/* Where the first bounded wait gave up since the last clear (0 if none): bit 31 set, site code in
 * bits 0-7 (kernel-specific), CTA index in bits 8-15, the waiting role's counter in bits 16-30.
 * Synchronises `stream`; clears when `clear` is non-zero.  For diagnosis of a KVB_DEV_TIMEOUT. */
kvb_status kvb_device_diag(unsigned* out, int clear, void* stream);

/* ------------------------------------------------------------------------------------------ *
 * K1: quantise + planar-pack.  Replaces kivi_quant (STRATA_KV.py:826-856), strata_quantize +
 * pack_planar (STRATA_KV.py:1158-1182) and the per-stratum gather of StrataMethod.pack
 * (STRATA_KV.py:1611-1627) / SnapKVQuantMethod.entries (STRATA_KV.py:1024-1027).
 *
 * Rows: for each (b, h), stored row j (0 <= j < n) is source row idx[b, h, j] when idx is given,
 * else source row first_row + j.  x: (B, H, T, d) of dtype x_dtype with element strides
 * (sb, sh, st) and unit channel stride.  bits in {2, 4, 8}; d % 32 == 0 and d <= 256.
 * Outputs (all dense, row capacity n_alloc >= n per (b, h); n_alloc % 16 == 0):
 *   codes (B, H, n_alloc, d * bits / 8) planar bytes (byte i holds channel p * d / P + i in bits
 *         [p * bits, (p + 1) * bits), P = 8 / bits);
 *   meta  ASYM per token:    (B, H, n_alloc, d / group, 2) fp16 (lo, scale) pairs;
 *         ASYM per channel:  (B, H, n_alloc / group, d, 2) fp16 (lo, scale) pairs, group in
 *                            {16, 32, 64, 128}; a partial last group uses its valid rows only
 *                            (the reference's repeat-last-row padding leaves min / max unchanged);
 *         MIDRISE:           (B, H, n_alloc) fp16 scales (group must equal d);
 *   xhat  optional (nullable) float32 (B, H, n, d): what a reader dequantises.
 * `step` is the MIDRISE step in RMS units (uniform_step(bits)[0], STRATA_KV.py:1133). */
/* As kvb_quant_pack in per-token mode (k_mode KVB_K_PER_TOKEN), with the codes written in the value
 * block layout read by the tensor-core decode: for every 128-token block of each (b, h), d rows
 * (one per channel) of 16 * bits bytes; byte k of channel row c holds the codes of tokens
 * p * 128 / P + k (P = 8 / bits) in bits [p * bits, (p + 1) * bits) - the planar packing applied
 * along tokens.  Codes, metadata and xhat are the same numbers kvb_quant_pack produces.  Needs
 * d == 128, fp16 / bf16 input with 16-byte aligned rows, n_alloc % 128 == 0, 16-byte aligned
 * meta.  No counterpart in the reference (an internal layout of this library's decode). */
kvb_status kvb_quant_pack_blocked(const void* x, int x_dtype, int64_t B, int64_t H, int64_t T, int64_t d,
                                  int64_t sb, int64_t sh, int64_t st, const int64_t* idx, int64_t first_row,
                                  int64_t n, int64_t n_alloc, int bits, int group, int code_kind, float step,
                                  uint8_t* codes, void* meta, float* xhat, void* stream);

kvb_status kvb_quant_pack(const void* x, int x_dtype, int64_t B, int64_t H, int64_t T, int64_t d,
                          int64_t sb, int64_t sh, int64_t st,
                          const int64_t* idx, int64_t first_row, int64_t n, int64_t n_alloc,
                          int bits, int group, int k_mode, int code_kind, float step,
                          uint8_t* codes, void* meta, float* xhat, void* stream);

/* ------------------------------------------------------------------------------------------ *
 * K2: rank split + compaction (budgeted eviction / strata assignment).  Replaces the topk + sort
 * of SnapKVQuantMethod.entries (STRATA_KV.py:1022-1023) and the importance ordering that feeds the
 * strata (STRATA_KV.py:1560-1571).  For each of `rows` rows of `n` keys (f32 or f64, row stride
 * key_stride elements), elements are ranked by key descending, ties by LOWER index first; class c
 * takes ranks [sum(counts[:c]), sum(counts[:c+1])) and the last class takes the rest
 * (n_classes <= 4, n_classes - 1 counts given).  out[c] (nullable) receives, per row, the class's
 * indices in ASCENDING order, row stride out_stride[c].  NaN keys are rejected by the wrapper. */
kvb_status kvb_rank_split(const void* keys, int key_dtype, int64_t rows, int64_t n, int64_t key_stride,
                          int n_classes, const int64_t* counts, int64_t* const* out,
                          const int64_t* out_stride, void* stream);

/* Per-token key energy sum_c k_c^2 in float64 (exact for bf16 / fp16 keys, so rankings are
 * order-independent): k (B, H, T, d) strides (sb, sh, st) -> out (B, H, T) float64. */
kvb_status kvb_key_energy(const void* k, int dtype, int64_t B, int64_t H, int64_t T, int64_t d,
                          int64_t sb, int64_t sh, int64_t st, double* out, void* stream);

/* Accumulated attention of `nq` queries per query head over all T keys (SnapKV-style scores,
 * snapkv_scores STRATA_KV.py:932-953 with decode-time queries): for each (b, kv head h),
 * score[j] = mean over the rep query heads and nq queries of softmax_j(scaling * q . k_j), for
 * j < n_cand; q (B, Hq, nq, d), k (B, Hkv, T, d) in dtype (f16 / bf16), dense, d in {64, 128},
 * rep * nq <= 256; out (B, Hkv, n_cand) float32.  `pool` in {0, 1, 3, 5, ...}: avg_pool1d over
 * the candidates (zero padding counted) before the head mean.  workspace: 256-byte aligned,
 * >= kvb_scores_workspace_size(B, Hkv, n_cand) bytes. */
size_t kvb_scores_workspace_size(int64_t B, int64_t Hkv, int64_t n_cand);
kvb_status kvb_query_scores(const void* q, const void* k, int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                            int64_t nq, int64_t T, int64_t d, float scaling, int64_t n_cand, int pool,
                            float* out, void* workspace, size_t workspace_bytes, void* stream);

/* SnapKV scores at the compression horizon, the reference's own mode (snapkv_scores
 * STRATA_KV.py:932-954): q (B, Hq, w, d) holds the queries of the last w context positions H - w ..
 * H - 1 (the observation window), k (B, Hkv, H, d) the context keys.  Window query i sees keys
 * j <= H - w + i (the causal triu mask of :946); its softmax runs over every key it sees, window
 * keys included; out (B, Hkv, H - w) float32 = the mean over the window queries and the group's
 * query heads of those probabilities for the candidate columns j < H - w, avg_pool1d(pool) as in
 * kvb_query_scores.  The window's own columns (the reference pads them with max + 1 so they are
 * always kept) are not written: the caller keeps the window.  Same dtypes, limits (rep * w <= 256)
 * and workspace (kvb_scores_workspace_size(B, Hkv, H - w)) as kvb_query_scores. */
kvb_status kvb_snapkv_scores(const void* q, const void* k, int dtype, int64_t B, int64_t Hq, int64_t Hkv,
                             int64_t w, int64_t H, int64_t d, float scaling, int pool, float* out, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------------ *
 * K4: spectral code.  Replaces the basis projection of spectral_side (QUASAR_KV.py:1354-1382, with a
 * fixed per-head orthonormal basis) followed by the per-token mid-rise code of strata_quantize
 * (STRATA_KV.py:1158-1168) on the leading r = 32 coefficients, on tcgen05 tensor cores.
 * x: (B, H, T, 128) fp16, unit channel stride, element strides sb / sh / st of batch, head and token
 * (multiples of 8, i.e. 16 bytes: any layout a model's K / V projection produces), 16-byte aligned.  basis_t: (2, H, 32, 128) fp16 = the transposed
 * leading basis columns split into a high part and a low part (basis = hi + lo to ~22 bits).
 * Outputs per kvb_quant_pack's mid-rise layout: codes (B, H, n_alloc, 32 * bits / 8) planar, scales
 * (B, H, n_alloc) fp16; coef (nullable) (B, H, T, 32) float32 coefficients.  `step`: the mid-rise
 * step in RMS units (uniform_step(bits)[0]).  n_ctas: persistent CTAs (0 = one per SM). */
kvb_status kvb_spectral_encode(const void* x, int64_t B, int64_t H, int64_t T, int64_t sb, int64_t sh, int64_t st,
                               const void* basis_t, int bits, float step, uint8_t* codes, void* scales,
                               int64_t n_alloc, float* coef, int n_ctas, void* stream);

/* ------------------------------------------------------------------------------------------ *
 * Sequence split across ranks over peer memory (one process per GPU on one NVLink / NVSwitch node).
 * Each rank allocates an exchange region (kvb_xchg_alloc, zero-initialised flags), shares its IPC
 * handle with the other ranks (any host channel, e.g. a torch.distributed all-gather of the 64
 * bytes) and maps theirs (kvb_xchg_open).  kvb_xchg_merge then replaces the all-gather of every
 * rank's (output, lse) part and the LSE merge (kvb_lse_merge) with one kernel: this rank's rows go
 * straight into every peer's region, a per-slice flag is published, and each slice is merged once
 * every rank's flag for it has arrived (bounded wait; KVB_DEV_TIMEOUT on expiry).  All ranks must
 * make the same sequence of calls with the same rows and d; the call count is kept on the device,
 * so the call can sit in a CUDA graph.  Plain stores into peer memory only. */
size_t kvb_xchg_bytes(int64_t rows, int d, int world);
kvb_status kvb_xchg_alloc(size_t bytes, void** region, unsigned char* handle /* 64 bytes out */);
kvb_status kvb_xchg_open(const unsigned char* handle /* 64 bytes */, void** region);
kvb_status kvb_xchg_close(void* peer_region);
kvb_status kvb_xchg_free(void* region);
/* Zero this rank's own region on `stream` (re-establishing the exchange after a timeout). */
kvb_status kvb_xchg_zero(void* region, size_t bytes, void* stream);
/* part (rows, d) float32 and lse (rows) float32: this rank's decode_lse output; regions: `world`
 * device pointers (this rank's own region at [rank], the mapped peers' elsewhere); out (rows, d).
 * timeout_ns bounds each wait for a peer's rows (0: 2 s).  A wait that runs out sets KVB_DEV_TIMEOUT
 * in the device status word (site 0x40 in kvb_device_diag) and the slice is merged from what arrived.
 * While the status word holds KVB_DEV_TIMEOUT no call does anything (site 0x41): re-establish the
 * exchange first - on every rank clear the status (kvb_device_status with clear), synchronise the
 * ranks, zero the whole region (its flags and call counters restart at 0), synchronise again. */
kvb_status kvb_xchg_merge(const float* part, const float* lse, int64_t rows, int d, int rank, int world,
                          void* const* regions, void* out, int out_dtype, uint64_t timeout_ns, void* stream);

/* ------------------------------------------------------------------------------------------ *
 * K5: per-vector row codes (token-like stored vectors and format variants).  Rows follow
 * kvb_quant_pack's convention: for each (b, h), stored row j < n is source row idx[b, h, j] when
 * idx is given, else first_row + j, of x (B, H, T, d) with element strides (sb, sh, st) and unit
 * channel stride.  Packed rows are MSB-first bit streams (code i in bits [i b, (i + 1) b), most
 * significant first), which for d * b % 8 == 0 is the reference's pack_codes of the row-major
 * codes (STRATA_KV.py:2728-2733). */
#define KVB_ABSMAX_STRATA 0   /* s = max(fp16(max|x| / qmax), 2^-24): absmax_quant STRATA_KV.py:549-554 */
#define KVB_ABSMAX_TILT 1     /* s = max(max|x|, 1e-8) / qmax in float32: fake_quant_tokens TILT_KV.py:721-727 */

/* Symmetric absmax code of every row, qmax = 2^(bits-1) - 1, codes clamp(rint(x / s), -qmax, qmax)
 * stored as codes + qmax (the bytes payload_bytes charges, STRATA_KV.py:2765-2766).  bits in 2..8,
 * d % 32 == 0, d <= 256.  packed (B, H, n, d * bits / 8); scale (B, H, n) float32 (an fp16 value
 * for KVB_ABSMAX_STRATA); xhat nullable (B, H, n, d) float32 = codes * s (what the reference's
 * fake_quant_tokens returns).  Replaces fake_quant_tokens of the chunk methods (STRATA_KV.py:557-564,
 * :587-591; TILT_KV.py:756-765). */
kvb_status kvb_absmax_quant(const void* x, int x_dtype, int64_t B, int64_t H, int64_t T, int64_t d,
                            int64_t sb, int64_t sh, int64_t st, const int64_t* idx, int64_t first_row, int64_t n,
                            int bits, int variant, uint8_t* packed, float* scale, float* xhat, void* stream);

/* MSB-first packing of `rows` rows of w codes (uint8, < 2^bits): out (rows, w * bits / 8); bits in
 * 1..8, w * bits % 8 == 0.  pack_rows QUASAR_KV.py:1185-1190, pack_codes STRATA_KV.py:2728. */
kvb_status kvb_pack_rows(const uint8_t* codes, int64_t rows, int64_t w, int bits, uint8_t* out, void* stream);

/* Table decode of MSB-first rows: out[r, i] = (accumulate ? out[r, i] : 0) + levels[code_i] (times
 * row_scale[r] when given), float32 (rows, w).  levels: 2^bits float32 on the device.  One call per
 * stage of an embedded code sums the stages in order (byte_lut QUASAR_KV.py:1194-1203,
 * embedded_quantize :1172-1182). */
kvb_status kvb_decode_rows_lut(const uint8_t* packed, int64_t rows, int64_t w, int bits, const float* levels,
                               const float* row_scale, int accumulate, float* out, void* stream);

/* HEDGE per-token code at d = 128 (hedge_quant / centered_code HEDGE_KV.py:1103-1130): y = (x - mu) R^T
 * (float32; mu nullable (H, 128) float32, R (128, 128) float32 row-major), then at bits 1..4 the
 * Lloyd-Max levels (2^bits float32, `levels`) times s = max(fp16(RMS(y)), 2^-24), codes =
 * bucketize(y / s, level midpoints); at bits 8 s = max(fp16(max|y| / 127), 2^-24), codes =
 * clamp(rint(y / s), -127, 127) + 127.  packed (B, H, n, 16 * bits) MSB-first; scale (B, H, n)
 * float32; y, xhat nullable (B, H, n, 128) float32, xhat = (level s) R + mu. */
kvb_status kvb_hedge_quant(const void* x, int x_dtype, int64_t B, int64_t H, int64_t T, int64_t sb, int64_t sh,
                           int64_t st, const int64_t* idx, int64_t first_row, int64_t n, const float* mu,
                           const float* R, int bits, const float* levels, uint8_t* packed, float* scale, float* y,
                           float* xhat, void* stream);

/* TILT chunk selection (finalize_chunk TILT_KV.py:743-760, eviction and tail part): for each of U x H
 * chunks of C <= 128 keys (k (U, H, C, 128), element strides su, sh, sc, unit channel stride) and
 * nq observed queries qref (U, H, nq, 128) float32 (already scaled), share[c] = mean over queries of
 * softmax_c(qref . k_c); idx (U, H, m) receives the m largest shares' positions (ties: lower
 * position first) in ascending order; share (U, H, C) nullable.  A NaN share sets KVB_DEV_NAN. */
kvb_status kvb_chunk_select(const void* k, int k_dtype, int64_t U, int64_t H, int64_t C, int64_t su, int64_t sh,
                            int64_t sc, const float* qref, int64_t nq, int64_t m, int64_t* idx, float* share,
                            void* stream);

/* ------------------------------------------------------------------------------------------ *
 * K3: fused split-K flash decode over a packed, head-synchronous cache.  Replaces StrataState.attend
 * + strata_tier_kernel (STRATA_KV.py:1762-1796, :1450-1469), LayerState.attend / chunked_attention
 * (STRATA_KV.py:716, :641) over KIVI codes, and QuasarState.attend (QUASAR_KV.py:1942-1967, one
 * stage) over spectral coefficients. */
#define KVB_V_TOKEN_MAJOR 0   /* value codes as kvb_quant_pack writes them */
#define KVB_V_BLOCK128 1      /* value codes as kvb_quant_pack_blocked writes them (tensor-core decode) */

typedef struct kvb_stratum {
    int kbits, vbits;         /* code widths of keys and values: 2, 4 or 8 each */
    int v_layout;             /* KVB_V_TOKEN_MAJOR or KVB_V_BLOCK128 */
    int reserved;             /* 0 */
    int64_t n;                /* stored tokens per (b, h) */
    int64_t n_alloc;          /* row capacity per (b, h), multiple of 16 (of 128 for KVB_V_BLOCK128) */
    const uint8_t* kc;        /* (B, Hkv, n_alloc, d_code * kbits / 8) planar */
    const uint8_t* vc;        /* token-major: (B, Hkv, n_alloc, d_code * vbits / 8) planar;
                               * block: (B, Hkv, n_alloc / 128, d_code, 16 * vbits) */
    const void* kmeta;        /* as kvb_quant_pack's meta for the key code */
    const void* vmeta;        /* as kvb_quant_pack's meta for the value code (per token) */
} kvb_stratum;

typedef struct kvb_cache {
    int B, Hkv;
    int d;                    /* model head dim (exact rows, queries, output) */
    int d_code;               /* coded dimension (== d, or r for the spectral code) */
    int code_kind;            /* KVB_CODE_ASYM / KVB_CODE_MIDRISE */
    int k_mode;               /* KVB_K_PER_TOKEN / KVB_K_PER_CHANNEL */
    int k_group;              /* channels per key group (per token) or tokens per group (per channel) */
    int v_group;              /* channels per value group */
    int n_strata;             /* 0..4 */
    kvb_stratum strata[4];
    /* exact rows (model dtype, (B, Hkv, cap, d) dense): rows [0, n0) always readable, rows
     * [n0, n_exact) sit at positions pos0 + (i - n0) (causal w.r.t. each query's position) */
    const void* k_exact;
    const void* v_exact;
    int exact_dtype;
    int64_t exact_cap, n_exact, n0, pos0;
    /* optional query map and output lift (code space != model space), float32:
     *   qmap (Hkv, d, d_code): q_code = q @ qmap[h]   (rotation R^T, or spectral basis B_r)
     *   lift (Hkv, d_code, d): out_code @ lift[h]     (R, or B_r^T)
     *   mu_k, mu_v (Hkv, d):   mean key / value (logit bias scaling q . mu_k; value (sum p) mu_v) */
    const float* qmap;
    const float* lift;
    const float* mu_k;
    const float* mu_v;
} kvb_cache;

/* Options of the kvb_decode* calls made afterwards on the calling host thread; returns the previous
 * options.  KVB_DECODE_OVERLAP: a call's main kernel may launch as a programmatic dependent of the
 * kernel before it on the stream and start copying the packed cache while that kernel finishes (q,
 * the workspace and the outputs are touched only after that kernel has completed).  Set it only when
 * the kernel launched immediately before each call writes none of the packed strata the call reads;
 * consecutive decode calls over a model's layers qualify.  Default: no options.  No counterpart in the
 * reference (eager PyTorch launches). */
#define KVB_DECODE_OVERLAP 1u
unsigned kvb_set_decode_flags(unsigned flags);

/* Number of split-K pieces and the plan / workspace sizes for a cache shape. */
size_t kvb_decode_workspace_size(const kvb_cache* c, int Hq, int Tq, int n_ctas);
/* q (B, Hq, Tq, d) dtype q_dtype dense; qpos (Tq) host array of query positions (used only for
 * appended exact rows); out (B, Tq, Hq, d) in out_dtype.  n_ctas: persistent CTAs (0 = one per
 * SM).  workspace: device buffer of kvb_decode_workspace_size bytes, 256-byte aligned, zero-filled
 * before its first use (e.g. one cudaMemsetAsync); every call leaves the part it needs zeroed again
 * (per-head counters of the in-kernel merge; a counter found non-zero sets KVB_DEV_WORKSPACE).
 * One kernel launch per call, except for the tcgen05 decode (block value layout) and caches of more
 * than 256 (batch, KV head) pairs, which add a query-prep and / or a merge kernel. */
kvb_status kvb_decode(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                      const int64_t* qpos, void* out, int out_dtype, int n_ctas,
                      void* workspace, size_t workspace_bytes, void* stream);

/* As kvb_decode, and records the cudaEvent_t handles ev_begin / ev_end (nullable) on `stream`
 * immediately before and after the main split-K kernel, so a caller can time that kernel alone. */
kvb_status kvb_decode_events(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                             const int64_t* qpos, void* out, int out_dtype, int n_ctas,
                             void* workspace, size_t workspace_bytes, void* stream, void* ev_begin, void* ev_end);

/* As kvb_decode, and also writes lse (B, Tq, Hq) float32: the natural-log sum of exp(scaled logit) over
 * every token this call attended (-inf, with a zero output row, where none was readable).  Used by
 * a sequence split: each rank decodes its own token range, the (out, lse) parts are exchanged, and
 * kvb_lse_merge combines them.  Replaces the per-stratum (m, l, acc) partials of strata_tier_kernel
 * (STRATA_KV.py:1450-1469) at the granularity of a whole rank. */
kvb_status kvb_decode_lse(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                          const int64_t* qpos, void* out, int out_dtype, float* lse, int n_ctas,
                          void* workspace, size_t workspace_bytes, void* stream);

/* Sequence-split decode with the cross-rank merge in the same kernel.  Each of `world` ranks (one GPU
 * each, peer access over NVLink / NVSwitch) holds a contiguous token range of every (batch, KV head)
 * in its cache c and calls this with the same q, shapes and order as the others; out (B, Tq, Hq, d)
 * receives attention over all ranks' tokens on every rank.  regions[r]: rank r's exchange region of
 * kvb_decode_xchg_bytes bytes (kvb_xchg_alloc on rank r, kvb_xchg_open of its handle elsewhere; zeroed
 * at allocation).  The CTA that merges a head writes this rank's normalised rows and lse into slot
 * `rank` of every region, publishes a flag per (rank, head), waits (bounded by timeout_ns, 0: 2 s) for
 * every rank's flag of the head and merges the parts with the arithmetic of kvb_lse_merge: one kernel
 * per call instead of kvb_decode_lse + kvb_xchg_merge.  A wait that runs out sets KVB_DEV_TIMEOUT
 * (site 0x42) and merges what arrived; while the status word holds it, calls write no output (site
 * 0x43) until the exchange is re-established as for kvb_xchg_merge (kvb_xchg_zero on every rank).
 * KVB_EUNSUPPORTED where the merge cannot run inside the main kernel (more than 256 (batch, KV head)
 * pairs, the tcgen05 value layout, an empty token range): use kvb_decode_lse + kvb_xchg_merge. */
size_t kvb_decode_xchg_bytes(const kvb_cache* c, int Hq, int Tq, int world);
kvb_status kvb_decode_xchg(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                           const int64_t* qpos, void* out, int out_dtype, int rank, int world,
                           void* const* regions, uint64_t timeout_ns, int n_ctas, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Merge of n_parts attention parts over disjoint token sets: part k's rows at parts + k * part_stride
 * ((rows, d) float32, each row normalised) with lse at lse + k * lse_stride ((rows) float32, natural
 * log).  out (rows, d) in out_dtype = sum_k exp(lse_k - M) o_k / sum_k exp(lse_k - M) (the exact LSE
 * merge of StrataState.attend, STRATA_KV.py:1784-1792, across parts).  Parts with lse -inf are
 * skipped; a row with no part gets zeros. */
kvb_status kvb_lse_merge(const float* parts, int64_t part_stride, const float* lse, int64_t lse_stride, int n_parts,
                         int64_t rows, int d, void* out, int out_dtype, void* stream);

/* Decode attention for callers that cannot allocate device memory.  No counterpart in the reference
 * (which allocates with PyTorch freely); added for hosts that hand an operator only its input and
 * output buffers: serving engines whose memory planner reserves all device memory up front and lets
 * no operator call cudaMalloc afterwards, and plugin interfaces that give an operator no allocator.
 * Same arguments and result as kvb_decode, minus the workspace: the split-K scratch lives in a
 * file-scope __device__ array of KVB_NOALLOC_SCRATCH_BYTES (8 MiB) that every device loading the
 * library keeps until process exit.  Requests needing more scratch return KVB_EINVAL (the message
 * gives the size needed; use kvb_decode with your own workspace for those).  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress, with that device current); make
 * that first call before any stream capture.  All calls share the one array.  Its per-head merge
 * counters must be zero when a call starts: the array is zero when the library loads and every call
 * leaves them at zero again (a non-zero counter sets KVB_DEV_WORKSPACE).  Calls that overlap on the GPU
 * (concurrent streams, or several host threads) race on it: serialise them.  The current device must be the device of `stream` (KVB_EINVAL
 * otherwise). */
#define KVB_NOALLOC_SCRATCH_BYTES (8u << 20)
kvb_status kvb_decode_noalloc(const kvb_cache* c, const void* q, int q_dtype, int Hq, int Tq, float scaling,
                              const int64_t* qpos, void* out, int out_dtype, int n_ctas, void* stream);

/* STRATA's head-synchronous rate allocation (head_sync_allocate, STRATA_KV.py:1308-1351) on the device.
 * Dsort (n, nlev) float32 row-major, device: the distortion (summed over KV heads) of giving rank
 * position j option l, columns drop | coded level 1 .. nlev - 2 | exact; cost (nlev) and fixed
 * (nlev - 1) host arrays: bits of option l over the heads, and the layer's fixed bits when the deepest
 * coded level used is c (0: none).  Minimises sum_j Dsort[j, l_j] subject to sum_j cost[l_j] +
 * fixed[c] <= budget by Lagrangian relaxation: `rounds` rounds (4 in the reference) of `grid` (32)
 * multipliers on a log scale over [e^-80, e^25], then the allocation at the smallest feasible one.
 * Outputs (device): choice (n) int32, cap (1) int32, bits (1) float64.  workspace: device buffer of
 * kvb_head_sync_allocate_workspace() bytes, 16-byte aligned (its round counter is reset by every
 * call).  No host synchronisation: rounds are launched back to back.  Choices equal the reference's
 * except where two layer totals agree to float32 rounding (totals are summed in float64 here). */
size_t kvb_head_sync_allocate_workspace(void);
kvb_status kvb_head_sync_allocate(const float* Dsort, int64_t n, int nlev, const float* cost, const float* fixed,
                                  double budget, int rounds, int grid, int32_t* choice, int32_t* cap, double* bits,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* QUASAR's coded decode over embedded stage codes: the sums of QuasarState.coded_scores / coded_values
 * (QUASAR_KV.py:1918-1940; its Triton kernels :1498-1556 compute the same).  flat (flat_bytes, device):
 * every step's (Hkv, n_s, bytes) block of MSB-first packed codes; table (n_steps x 7 int32, HOST):
 * offset, n_s, bytes per row, band start a, band width w, bits b, level offset; levels (n_levels
 * float32, HOST): the stage level tables, concatenated.  Step s owns tokens [0, n_s) and coefficients
 * [a, a + w).  scores (Hkv, rows, n_c) = sum over owning steps of qt[band] . level[codes], from qt
 * (Hkv, rows, R); values (Hkv, rows, R) = sum_j pv[j] level[codes] per band, from pv (Hkv, rows, n_c),
 * without atomics (token splits added in a fixed order; workspace of kvb_quasar_values_workspace
 * bytes).  rows <= 32, R <= 256, n_steps <= 32, n_levels <= 64; float32 device tensors, dense. */
kvb_status kvb_quasar_scores(const float* qt, int Hkv, int rows, int R, const uint8_t* flat, size_t flat_bytes,
                             const int32_t* table, int n_steps, const float* levels, int n_levels, int64_t n_c,
                             float* scores, void* stream);
size_t kvb_quasar_values_workspace(int Hkv, int rows, int64_t n_c, int R);
kvb_status kvb_quasar_values(const float* pv, int Hkv, int rows, int64_t n_c, const uint8_t* flat, size_t flat_bytes,
                             const int32_t* table, int n_steps, const float* levels, int n_levels, int R,
                             float* values, void* workspace, size_t workspace_bytes, void* stream);

/* TILT's moment atoms of a chunk's bulk (moment_atoms, TILT_KV.py:622-670, built by the caller), float32
 * device tensors, dense: mu_k (B, Hkv, NA, d), logn (B, Hkv, NA), U (B, Hkv, NA, d, r), lam (B, Hkv, NA, r),
 * diag (B, Hkv, NA, d), R (B, Hkv, NA), A (B, Hkv, NA, d, r), Bk (B, Hkv, NA, d, r), Rv (B, Hkv, NA);
 * the tensors the flags do not use may be null. */
typedef struct kvb_atoms {
    const float* mu_k;
    const float* logn;
    const float* U;
    const float* lam;
    const float* diag;
    const float* R;
    const float* A;
    const float* Bk;
    const float* Rv;
    int B, Hkv, NA, d, r;     /* d <= 256, 1 <= r <= 8 */
    int order, tilt, project, phase;
} kvb_atoms;

/* atom_read (TILT_KV.py:673-714): for scaled queries qs (B, Hq, c, d) float32, the logit and value
 * factor of every (query, atom) pair, logit / cfac (B, Hq, c, NA), and with tilt the coordinates tB
 * (B, Hq, c, NA, r); KV head h serves query heads h * rep .. (HF repeat_kv order). */
kvb_status kvb_atom_read(const kvb_atoms* m, const float* qs, int Hq, int c, float* logit, float* cfac, float* tB,
                         void* stream);

/* STRATA's coverage statistics of one layer (coverage_stats, STRATA_KV.py:1226-1298; replaces the
 * reference's eager torch code called from StrataMethod.compress_layer, :1537).  q (Hq, H, d) (only the
 * rows at the groups' positions are read), k and v (Hkv, H, d), all three of `dtype` with d contiguous
 * and the element strides below (multiples of 16 bytes); M (Hq, d, d) float32 dense, M_a = W_O,aᵀ W_O,a
 * (:1519-1526).  The observation groups (coverage_groups, :1206-1222, computed by the caller; pass the
 * last alone for window_only) are the host arrays pos[group_off[g] .. group_off[g + 1]); the last group
 * counts reads at any distance >= 1, the others at distance >= local.  Outputs, float32 device
 * tensors: A, W, DD (Hkv, re - rs), S and Mbar (Hkv, d, d).  d in {64, 128}; Hq / Hkv <= 8. */
typedef struct kvb_coverage {
    const void* q;
    const void* k;
    const void* v;
    int dtype;                          /* KVB_F32 / KVB_F16 / KVB_BF16 for q, k and v */
    int64_t q_head_stride, q_pos_stride, kv_head_stride, kv_pos_stride;
    const float* M;
    int Hq, Hkv, d;
    int64_t H, rs, re;                  /* context length; coded tokens [rs, re) */
    float scaling;                      /* query scale */
    float floor;                        /* STRATA_FLOOR */
    int local;                          /* STRATA_LOCAL */
    int64_t score_cap;                  /* bytes of stored scores per pass over a batch of groups; 0: 4 GiB */
} kvb_coverage;
/* Device workspace bytes of kvb_coverage_stats for these groups (0 for invalid arguments). */
size_t kvb_coverage_workspace_size(const kvb_coverage* c, const int64_t* pos, const int64_t* group_off, int n_groups);
kvb_status kvb_coverage_stats(const kvb_coverage* c, const int64_t* pos, const int64_t* group_off, int n_groups,
                              float* A, float* W, float* DD, float* S, float* Mbar, void* workspace,
                              size_t workspace_bytes, void* stream);

/* LCTC's clipped uniform quantiser (uq_codes / uq_values, LCTC_KV.py:443-455): per column k a width
 * bits[k] (integral, 1..8) and a clip; code = min(max(floor((a + clip) / step), 0), 2^bits - 1) with
 * step = 2 clip / 2^bits, value = -clip + (code + 0.5) step, each operation rounded as float32 (codes and
 * values bit-identical to the reference).  a (rows, n) float32 with row stride lda; codes (rows, n) uint8
 * and values (rows, n) float32 dense (values may be null). */
kvb_status kvb_uq_codes(const float* a, int64_t rows, int64_t n, int64_t lda, const float* bits, const float* clip,
                        uint8_t* codes, float* values, void* stream);
kvb_status kvb_uq_values(const uint8_t* codes, int64_t rows, int64_t n, int64_t ldc, const float* bits,
                         const float* clip, float* values, void* stream);
/* operational_rd (LCTC_KV.py:458-481): per column of A (rows = calibration tokens) D[k][0] = mean a^2 and,
 * per width bits_set[j] (host array, bits_set[0] = 0, the others 1..8, nb <= 16), the least mean squared
 * quantisation error over the clips mults[m] x rms (mults: n_mults float32 on the device, the reference's
 * logspace(0.5, 8)), the first on ties, and that clip: D (n, nb) float64, C (n, nb) float32. */
size_t kvb_operational_rd_workspace(int64_t n, int nb, int n_mults);
kvb_status kvb_operational_rd(const float* A, int64_t rows, int64_t n, int64_t lda, const int32_t* bits_set, int nb,
                              const float* mults, int n_mults, double* D, float* C, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Build the split-K plan (pure host computation, no CUDA calls) for n_ctas CTAs.  plan_out receives
 * [n_ctas, n_pieces, n_heads, cta_begin[n_ctas + 1], n_pieces x (head, stratum, first chunk, end
 * chunk, slot), head_begin[n_heads + 1]]: pieces in CTA order, each with the slot of its partial;
 * slots are head-major and head_begin indexes them.  Returns the number of int32 needed (the table
 * is written only when plan_capacity suffices).  Exposed for tests; kvb_decode builds it itself. */
int64_t kvb_decode_plan(const kvb_cache* c, int n_ctas, int32_t* plan_out, int64_t plan_capacity);

#ifdef __cplusplus
}
#endif
#endif /* KVB_H */
