/*
 * fgg_api.h - C ABI of the B200 (sm_100a) block-scaled FP4 grouped GEMM.
 *
 * Every entry point takes plain pointers and sizes; no framework types cross
 * this boundary.  Device buffers are owned by the caller.  Calls are
 * stream-ordered on the `stream` argument (a cudaStream_t passed as void*,
 * NULL = legacy default stream) and never synchronise the host, except
 * fgg_read_device_status, which exists to do exactly that.
 *
 * Two operator families share one tcgen05 engine:
 *
 *  1. NVFP4 x NVFP4 grouped GEMM with per-group operand lists (the operator
 *     the benchmark configs describe).  Semantics, for every group g:
 *        C_g[m, n] = alpha_g * sum_k deq(A_g)[m, k] * deq(B_g)[n, k]
 *        deq(X)[r, k] = e2m1(code(X, r, k)) * e4m3(sf(X)[r, k / 16])
 *     with codes packed two per byte (element 2j in the LOW nibble of byte j),
 *     one E4M3 scale per 16 contiguous K elements, fp32 accumulation, bf16
 *     output.  alpha_g is the product of the two per-tensor fp32 global
 *     (decode) scales.  The reference repository has no NVFP4 Blackwell kernel;
 *     these entry points replace the operator described by its benchmark card
 *     and restate the NVFP4 decode used by
 *     tasks/muse_prefill_boundary/reference/submission.py:538-549 and :1847-1880
 *     (e2m1 code x e4m3 block scale x fp32 global scale).
 *
 *  2. MXFP8 x MXFP4 M-grouped GEMM with contiguous grouping (m_indices), the
 *     exact operator of kernels/gemm/fp4_grouped_gemm/b200/kernel.py:2788-2862
 *     (`fp4_grouped_gemm(a, a_sf, b, b_sf, m_indices) -> c`).
 *
 * Return codes are FGG_OK (0) or one of the FGG_E* values below;
 * fgg_last_error_detail() gives a message for the calling thread's last
 * failure.
 */
#ifndef FGG_API_H
#define FGG_API_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FGG_API __attribute__((visibility("default")))
#else
#define FGG_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FGG_OK = 0,
  FGG_EINVAL = 1,      /* null pointer, negative size, too many groups        */
  FGG_EBADSHAPE = 2,   /* N % 128 != 0, K % 64 != 0, K < 64, ...               */
  FGG_EALIGN = 3,      /* a device pointer is not 16-byte aligned             */
  FGG_EWORKSPACE = 4,  /* workspace / weight pack smaller than required        */
  FGG_ECUDA = 5,       /* a CUDA runtime call failed                           */
  FGG_ETIMEOUT = 6,    /* a device-side wait hit its time limit (see status)   */
  FGG_EARCH = 7        /* the current device is not an sm_100 part             */
};

/* Largest number of groups one call accepts (per-group metadata travels as
 * kernel parameters). */
#define FGG_MAX_GROUPS 512

FGG_API const char* fgg_error_string(int code);
FGG_API const char* fgg_last_error_detail(void);
/* Library build identifier ("fgg <version> sm_100a"). */
FGG_API const char* fgg_version(void);

/* ------------------------------------------------------------------------ */
/* NVFP4 x NVFP4 grouped GEMM                                                */
/* ------------------------------------------------------------------------ */

/* Expert / group weights.  B_g codes: [N, K/2] uint8, row-major.  B_g scales:
 * [N, K/16] E4M3 bytes, row-major.  All groups share N and K. */
typedef struct FggNvfp4Weights {
  int32_t num_groups;
  int32_t n;
  int32_t k;
  const void* const* b;     /* host array [G] of device pointers */
  const void* const* b_sf;  /* host array [G] of device pointers */
} FggNvfp4Weights;

/* Size of the device buffer fgg_nvfp4_pack_weights fills: per-group TMA
 * descriptors plus the scales repacked into the MMA's 512-byte SF atoms.
 * Replaces the identity-cached host repack `_prepare` / `_pack_sf_wgt` of
 * kernels/gemm/fp4_grouped_gemm/b200/kernel.py:2709-2786, done on the device. */
FGG_API size_t fgg_nvfp4_weight_pack_bytes(int32_t num_groups, int32_t n, int32_t k);
FGG_API int fgg_nvfp4_pack_weights(const FggNvfp4Weights* w, void* pack, size_t pack_bytes,
                           void* stream);

/* One grouped GEMM call.  A_g codes [M_g, K/2] uint8; A_g scales [M_g, K/16]
 * E4M3; alpha: device fp32 [G]; out: device bf16 [sum_g M_g, N] where group g
 * occupies rows [sum_{h<g} M_h, sum_{h<=g} M_h).  M_g may be 0. */
typedef struct FggNvfp4Problem {
  int32_t num_groups;
  int32_t n;
  int32_t k;
  const int32_t* m;         /* host array [G] */
  const void* const* a;     /* host array [G] of device pointers */
  const void* const* a_sf;  /* host array [G] of device pointers */
  const float* alpha;       /* device array [G] */
  void* out;                /* device bf16 */
  /* Optional: host array [G], the weight group (in `pack`) problem group g
   * multiplies with; NULL = group g uses weight group g.  Lets several
   * problem groups (e.g. the per-source chunks of one expert after an
   * all-to-all dispatch) share one packed weight group. */
  const int32_t* b_index;
  int32_t num_weight_groups; /* groups in `pack` when b_index is set */
} FggNvfp4Problem;

/* Scratch the call needs (token-scale repack, per-group descriptors, tile
 * list, status words).  Replaces the per-call part of `_prepare`
 * (kernels/gemm/fp4_grouped_gemm/b200/kernel.py:2751-2786). */
FGG_API size_t fgg_nvfp4_workspace_bytes(const FggNvfp4Problem* p);
/* Replaces `fp4_grouped_gemm` (kernel.py:2788-2862) for the NVFP4 format:
 * validates, repacks the token scales, builds descriptors and launches the
 * persistent tcgen05 kernel.  `pack` must come from fgg_nvfp4_pack_weights
 * for the same N, K and G weight groups (num_weight_groups when b_index is
 * set). */
FGG_API int fgg_nvfp4_grouped_gemm(const FggNvfp4Problem* p, const void* pack, void* workspace,
                           size_t ws_bytes, void* stream);
/* The same GEMM with the gated epilogue of a fused gate+up projection: the
 * packed weight rows (N = 2I of them) come in 32-row chunks of 16 gate rows
 * then the 16 up rows of the same outputs; out is bf16 [sum_g M_g, N/2] with
 *   out[t, 16c + i] = bf16(silu(alpha_g * acc[t, 32c + i]) * alpha_g * acc[t, 32c + 16 + i]).
 * N % 32 == 0; workspace as for fgg_nvfp4_grouped_gemm.  No counterpart in
 * the reference operator: it is the SiLU * up epilogue of the gated expert
 * GEMM in tasks/muse_prefill_boundary/reference/submission.py:31-33 (fused
 * kernel) and :1096 (its self-test: silu(hh[:, :D]) * hh[:, D:]). */
FGG_API int fgg_nvfp4_grouped_gemm_silu_mul(const FggNvfp4Problem* p, const void* pack,
                                            void* workspace, size_t ws_bytes, void* stream);
/* The two halves of fgg_nvfp4_grouped_gemm, for callers that replay one
 * problem (same pointers, same sizes) many times, e.g. inside a CUDA graph:
 * fgg_nvfp4_prepare fills `workspace` (descriptors, token-scale repack, tile
 * list); fgg_nvfp4_gemm launches the GEMM kernel on a prepared workspace and
 * may be repeated.  The token scales must not change between the two. */
FGG_API int fgg_nvfp4_prepare(const FggNvfp4Problem* p, void* workspace, size_t ws_bytes, void* stream);
FGG_API int fgg_nvfp4_gemm(const FggNvfp4Problem* p, const void* pack, void* workspace, size_t ws_bytes,
                   void* stream);

/* The grouped GEMM over contiguous token rows with the group sizes in device
 * memory: the reference operator's own M-grouped layout (one concatenated
 * activation tensor, kernels/gemm/fp4_grouped_gemm/b200/kernel.py:10-37,
 * :2788-2795) in the NVFP4 format, with per-group offsets instead of a per-row
 * expert id.  Group g owns rows [offsets[g], offsets[g+1]) of a, a_sf and
 * out; the offsets may be written by an earlier kernel on the same stream
 * (e.g. an expert-parallel dispatch plan): the host never reads them, so a
 * call needs no host synchronisation and its host cost does not grow with G.
 * Rows outside every group are neither read for any output nor written.
 * Malformed offsets (decreasing, negative, past max_rows) run no tile and
 * leave status 0x203 in the workspace. */
typedef struct FggNvfp4RowsProblem {
  int32_t num_groups;
  int32_t n;
  int32_t k;
  int32_t max_rows;          /* rows allocated in a, a_sf, out, row_scale        */
  const int32_t* offsets;    /* device int32 [G + 1], nondecreasing, <= max_rows */
  const void* a;             /* device [max_rows, K/2] codes                     */
  const void* a_sf;          /* device [max_rows, K/16] E4M3 scales              */
  const float* alpha;        /* device fp32 [G]                                  */
  void* out;                 /* device bf16 [max_rows, N]                        */
  /* Optional device fp32 [max_rows]: a per-row factor applied with alpha,
   * out[r, n] = bf16(alpha_g * row_scale[r] * acc) (e.g. the per-source decode
   * scale of rows gathered from several ranks); NULL = 1. */
  const float* row_scale;
  /* Optional device int32 [G]: the packed weight group of problem group g
   * (NULL = g); a value outside [0, num_weight_groups) stops the kernel with
   * status 0x202 before any load of that tile. */
  const int32_t* b_index;
  int32_t num_weight_groups; /* groups in `pack` when b_index is set             */
  /* Optional host bound on every group's rows (0 = max_rows): at most 16
   * selects the decode tiles (16 tokens, weights streamed once). */
  int32_t max_group_rows;
} FggNvfp4RowsProblem;

FGG_API size_t fgg_nvfp4_rows_workspace_bytes(const FggNvfp4RowsProblem* p);
FGG_API int fgg_nvfp4_grouped_gemm_rows(const FggNvfp4RowsProblem* p, const void* pack,
                                        void* workspace, size_t ws_bytes, void* stream);

/* No counterpart in the reference (its operator always allocates its scale
 * repack and outputs through torch).  fgg_nvfp4_grouped_gemm for callers that
 * cannot allocate device memory at call time: a serving loop that owns a
 * fixed memory budget, or a host without an allocator on the call path.  The
 * call runs the same kernels with its scratch in a fixed device array inside
 * this library (FGG_NOALLOC_SCRATCH_BYTES per device) instead of a caller
 * workspace; after its set-up (below) it allocates nothing: no cudaMalloc /
 * cudaFree and no allocating library call, and its host-side bookkeeping
 * lives in fixed arrays.
 *   - Limit: a problem whose fgg_nvfp4_workspace_bytes exceeds
 *     FGG_NOALLOC_SCRATCH_BYTES is refused with FGG_EWORKSPACE before any
 *     device work (use fgg_nvfp4_grouped_gemm with a caller workspace).
 *   - Nothing in the scratch has to start at zero: every call rewrites its
 *     status words and tile counters before the GEMM kernel reads them, and
 *     writes every other byte it later reads.
 *   - One scratch per device, shared by every call on that device: calls
 *     whose device work overlaps in time (different streams, or host threads
 *     without ordering between them) corrupt each other.  Issue them on one
 *     stream, or order them with events.
 *   - The first call on each device (more exactly, on each CUDA context: the
 *     array's address belongs to the context that loaded it, so a context
 *     created after cudaDeviceReset repeats this) performs one-time set-up:
 *     the scratch array's address via cudaGetSymbolAddress, which also loads
 *     its module and so reserves the array's device memory, and the kernels'
 *     shared-memory attribute.  The first call on each host thread also sets
 *     up that thread's parameter block (thread-local storage, which the C
 *     library may allocate on a thread's first use).  Make one warm-up call
 *     per device and per calling thread at initialisation, before any stream
 *     capture; later calls allocate nothing.
 *   - status_out: optional device pointer to one int32; when non-null the call
 *     ends with a stream-ordered copy of the device status word there
 *     (0 = clean; non-zero = a bounded wait gave up), since the scratch that
 *     holds it is not visible to the caller. */
#define FGG_NOALLOC_SCRATCH_BYTES (32u << 20)
FGG_API int fgg_nvfp4_grouped_gemm_noalloc(const FggNvfp4Problem* p, const void* pack,
                                           void* status_out, void* stream);

/* ------------------------------------------------------------------------ */
/* MXFP8 x MXFP4 contiguous M-grouped GEMM (reference operator)              */
/* ------------------------------------------------------------------------ */

/* Mirrors kernel.py:2788-2795 argument for argument:
 *   a         [M_total, K]     float8_e4m3fn
 *   a_sf      [M_total, K/128] fp32, powers of two (UE8M0-representable)
 *   b         [G, N, K/2]      uint8, packed e2m1 pairs
 *   b_sf      [G, N, K/32]     fp32, powers of two
 *   m_indices [M_total]        int32 expert id per row, -1 = padding
 *   c         [M_total, N]     bf16 output
 * Every expert segment starts at a multiple of 224 rows (kernel.py:28-33).
 * Shape rules follow kernel.py:2808-2824: N % 128 == 0, K % 128 == 0. */
typedef struct FggMxProblem {
  int32_t m_total;
  int32_t n;
  int32_t k;
  int32_t num_groups;
  const void* a;
  const float* a_sf;
  const void* b;
  const float* b_sf;
  const int32_t* m_indices;
  void* c;
  /* 1: `workspace` already holds the repacked scales and tile list of an
   * earlier call on the same a_sf / b_sf / m_indices (the identity-keyed cache
   * of kernel.py:2743-2786); the call then launches the GEMM alone. */
  int32_t reuse_prepared;
} FggMxProblem;

/* Scratch for the MX call (repacked UE8M0 scales, block->expert table,
 * descriptors, status): kernel.py:2679-2786 done on the device per call. */
FGG_API size_t fgg_mx_workspace_bytes(const FggMxProblem* p);
FGG_API int fgg_mx_grouped_gemm(const FggMxProblem* p, void* workspace, size_t ws_bytes,
                        void* stream);

/* ------------------------------------------------------------------------ */
/* Expert-parallel MoE: the byte-moving kernels around the grouped GEMM      */
/* ------------------------------------------------------------------------ */

/* Dispatch plan: a stable counting sort of the num_tokens x topk routes
 * (device topk_ids, row-major) by destination bin = owner[e] * local +
 * slot[e] (device int32 arrays over the num_experts <= 8192 experts; local =
 * experts per rank, world x local <= 512).  Writes counts[bin] (routes per bin),
 * src_row[p] (the token of the route at sorted position p) and route_pos[i]
 * (the sorted position of route i).  Within a bin the routes keep their
 * order, as a stable sort leaves them.  An expert id outside
 * [0, num_experts) sets *bad and gets route_pos -1.  Replaces the plan half
 * of `moe_gather_plan` (submission.py:843-895) and an argsort + bincount. */
FGG_API int fgg_moe_plan(const int32_t* topk_ids, int32_t num_tokens, int32_t topk,
                         const int32_t* owner, const int32_t* slot, int32_t num_experts,
                         int32_t world, int32_t local, int32_t* counts, int32_t* src_row,
                         int32_t* route_pos, int* bad, void* stream);
/* Dispatch gather: out row r = source row src_row[r] of both NVFP4 tensors
 * (codes [rows_in, code_bytes], scales [rows_in, sf_bytes]).  Row sizes and
 * pointers must be multiples of 4 bytes (16 for the vector path).  A source
 * index outside [0, rows_in) is skipped and sets *bad (device int) to 1.
 * Replaces the row gather of `moe_gather_plan`
 * (tasks/muse_prefill_boundary/reference/submission.py:843-895). */
FGG_API int fgg_moe_gather_rows(const void* codes, const void* sf, int64_t rows_in,
                                int32_t code_bytes, int32_t sf_bytes, const int32_t* src_row,
                                int64_t num_rows, void* out_codes, void* out_sf, int* bad,
                                void* stream);
/* Combine: out[t, :] = bf16(sum_k weights[t, k] * rows[route_row[t*topk + k], :])
 * with fp32 accumulation; rows bf16 [num_rows, n], n % 8 == 0, 16-byte
 * aligned.  A route row outside [0, num_rows) is skipped and sets *bad.
 * Replaces `moe_combine` (submission.py:843-895: weight the rows, sum them
 * back per token). */
FGG_API int fgg_moe_combine(const void* rows, int64_t num_rows, const int32_t* route_row,
                            const float* weights, int32_t num_tokens, int32_t topk, int32_t n,
                            void* out, int* bad, void* stream);

/* The expert-parallel layer without a host synchronisation.  No counterpart
 * in the reference's code (it has no distributed path); the single-GPU
 * analogue is `_moe_forward` (tasks/muse_prefill_boundary/reference/
 * submission.py:843-895: gather plan, grouped expert GEMM, weighted combine).
 * A dispatch buffer that can never overflow gives every (source, destination)
 * pair room for all of the source's tokens, which is the byte count of an
 * all-gather of the tokens: so each rank packs its tokens into records
 * (fgg_moe_pack_tokens), the ranks all-gather them, each rank expands the
 * routes of its own experts into expert-ordered rows (fgg_moe_expand), runs
 * fgg_nvfp4_grouped_gemm_rows on them with the
 * plan's offsets, sums every token's local routes with its router weights
 * (fgg_moe_reduce) and the ranks exchange those partial rows with an
 * equal-split all-to-all that each rank sums (fgg_moe_sum_partials).  All
 * sizes stay on the device.
 *
 * Tokens are described by strided views so that one set of kernels reads a
 * caller's own tensors or the gathered records alike; strides are in bytes. */
typedef struct FggMoeTokens {
  int32_t num_tokens;
  int32_t topk;
  int32_t k;                 /* hidden size: codes K/2 bytes, scales K/16 bytes */
  const void* codes;         int64_t codes_stride;
  const void* sf;            int64_t sf_stride;
  const int32_t* ids;        int64_t ids_stride;      /* topk expert ids per token  */
  const float* weights;      int64_t weights_stride;  /* topk router weights; NULL = 1 */
  const float* scale;        int64_t scale_stride;    /* decode scale; stride 0 = one */
  /* Double-buffered views (the peer exchange below): when epoch is non-NULL
   * every pointer above is advanced by ((*epoch + 1) & 1) * parity_bytes on
   * the device, so a view captured in a CUDA graph follows the forward's
   * buffer half.  NULL / 0 for a plain view. */
  const int64_t* epoch;      int64_t parity_bytes;
} FggMoeTokens;

/* Bytes of one token record: codes, scales, ids, weights, decode scale,
 * padded to 16 bytes (0 for a bad geometry). */
FGG_API size_t fgg_moe_record_bytes(int32_t k, int32_t topk);
/* Write one record per token into `records` (device, 16-byte aligned). */
FGG_API int fgg_moe_pack_tokens(const FggMoeTokens* tokens, void* records, void* stream);
/* Host-only: a view of `num_tokens` consecutive records as FggMoeTokens. */
FGG_API int fgg_moe_records_view(const void* records, int32_t num_tokens, int32_t k, int32_t topk,
                                 FggMoeTokens* out);
/* The routes of this rank's experts as expert-ordered token rows:
 * offsets[0..local] (device) place the routes of local expert s (its slot) at
 * rows [offsets[s], offsets[s+1]) of out_codes [max_rows, K/2] / out_sf
 * [max_rows, K/16]; route_row[t*topk + k] is route (t, k)'s row or -1
 * (another rank's expert, or an absent route: expert id < 0, as on the
 * padding tokens of a fixed-capacity dispatch); src_token[row] and
 * row_scale[row] (the token's decode scale) describe each row.  counts:
 * device scratch of 2 * local int32.  An expert id >= num_experts sets
 * *bad = 1; more routes than max_rows sets *bad = 2 (the excess is dropped).
 * local <= 1024.  Rows are placed by atomics, so their order inside an
 * expert may change from call to call; fgg_moe_reduce sums them back in
 * route order, so its output does not. */
FGG_API int fgg_moe_expand(const FggMoeTokens* tokens, const int32_t* owner, const int32_t* slot,
                           int32_t num_experts, int32_t rank, int32_t local, int32_t max_rows,
                           int32_t* counts, int32_t* offsets, int32_t* route_row,
                           int32_t* src_token, float* row_scale, void* out_codes, void* out_sf,
                           int* bad, void* stream);
/* out[t, :] = bf16(sum_k weights[t, k] * rows[route_row[t*topk + k], :]) over
 * the routes with a row (>= 0), fp32 accumulation; zeros for a token with
 * none.  rows bf16 [num_rows, n]; n % 8 == 0. */
FGG_API int fgg_moe_reduce(const void* rows, int32_t num_rows, const int32_t* route_row,
                           const FggMoeTokens* tokens, int32_t n, void* out, int* bad,
                           void* stream);
/* out[t, :] = bf16(sum_s parts[s * per_source + t, :]) in fp32 for t < tokens:
 * the partial rows every rank returned for this rank's tokens (per_source =
 * the dispatch capacity per rank). */
FGG_API int fgg_moe_sum_partials(const void* parts, int32_t world, int32_t per_source,
                                 int32_t tokens, int32_t n, void* out, void* stream);

/* The same exchange without NCCL: kernels that store straight into the
 * other ranks' buffers over NVLink (peer memory shared through CUDA IPC, no
 * multicast), fused with the byte work on either side of the exchange.
 * Arrival is signalled by epoch-tagged flags in each destination's memory,
 * written with release semantics after the data; every wait for them is
 * bounded (wait_ms, default 10 s), after which the waiter sets
 * *status = 0x301 and returns (its data is then incomplete).  The dispatch buffer is double
 * buffered on the forward's epoch parity, so one forward's stores never
 * touch the half a slower peer still reads.  The combine pulls: each rank
 * writes its partial rows into its own return buffer and each token's rank
 * reads them from there over NVLink; a rank overwrites that buffer only
 * after every rank has dispatched the next forward, i.e. finished reading
 * it.  No counterpart in the reference (it has no distributed code).
 *
 * Buffers (every rank allocates its own with fgg_peer_alloc and maps the
 * others' with fgg_peer_export / fgg_peer_import):
 *   gathered  [2][world * capacity][record bytes]   dispatch destination
 *   recv      [world * capacity][n] bf16             partial rows, read by their token's rank
 *   flags     [2][8] uint64 (arrivals: [0] dispatch, [1] combine, by source)
 * epoch (int64), counters (3 x int32), status (int32) and routes
 * ([capacity] int32) are this rank's own.  A token's record and partial row
 * travel only between its rank and the ranks that own one of its experts
 * (owner[e] of num_experts): routes[t] keeps that set of ranks, as a bit
 * mask, from the dispatch to the sum.  world <= 8. */
#define FGG_PEERS_MAX 8
typedef struct FggMoePeers {
  int32_t world;
  int32_t rank;
  int32_t capacity;          /* token slots per rank (the same on every rank) */
  int32_t n;                 /* output columns */
  int64_t* epoch;
  int32_t* counters;
  int* status;
  void* gathered[FGG_PEERS_MAX];  /* each rank's buffer, as mapped in this process */
  void* recv[FGG_PEERS_MAX];
  void* flags[FGG_PEERS_MAX];
  const int32_t* owner;      /* [num_experts] rank of each expert (device) */
  int32_t num_experts;
  int32_t* routes;           /* [capacity] destination ranks of each token, bit mask */
  int32_t wait_ms;           /* limit of each flag wait; 0 = 10000 (the waits span the
                                other ranks' host work as well as their kernels) */
} FggMoePeers;

FGG_API int fgg_peer_alloc(size_t bytes, void** ptr);
FGG_API int fgg_peer_free(void* ptr);
FGG_API size_t fgg_peer_handle_bytes(void);
FGG_API int fgg_peer_export(const void* ptr, void* handle);
FGG_API int fgg_peer_import(const void* handle, void** ptr);
FGG_API int fgg_peer_close(void* ptr);
/* Dispatch: this rank's tokens (num_tokens <= capacity) become records in
 * slots [rank * capacity, ...) of the gathered buffer of every rank that owns
 * one of the token's experts; the other ranks' slots get expert ids -1 only,
 * as do slots past num_tokens.  routes[t] = those ranks; then the arrival
 * flags. */
FGG_API int fgg_moe_dispatch_peers(const FggMoeTokens* tokens, const FggMoePeers* peers,
                                   void* stream);
/* Wait (bounded) until every rank's arrival flag of `kind` (0 dispatch,
 * 1 combine) carries this forward's epoch. */
FGG_API int fgg_moe_wait_peers(const FggMoePeers* peers, int32_t kind, void* stream);
/* fgg_moe_reduce into this rank's own recv buffer: the partial row of
 * gathered slot t (of world * capacity) in row t, for the tokens with a
 * route on this rank only, followed by the combine arrival flags. */
FGG_API int fgg_moe_reduce_peers(const void* rows, int32_t num_rows, const int32_t* route_row,
                                 const FggMoeTokens* tokens, const FggMoePeers* peers, int* bad,
                                 void* stream);
/* out[t, :] = bf16(sum_s recv_s[rank * capacity + t, :]) in fp32 for
 * t < tokens over the ranks s in routes[t], read from rank s's recv buffer
 * (zeros for a token with no route); then the epoch advances. */
FGG_API int fgg_moe_sum_peers(const FggMoePeers* peers, int32_t tokens, void* out, void* stream);

/* ------------------------------------------------------------------------ */
/* NVFP4 quantisation (activations and weights)                              */
/* ------------------------------------------------------------------------ */

/* amax of |x| over `count` elements into *amax_out (device fp32).
 * x_dtype: 0 = fp32, 1 = bf16. */
FGG_API int fgg_amax(const void* x, int32_t x_dtype, int64_t count, float* amax_out, void* stream);

/* Quantise a row-major [rows, k] tensor to NVFP4:
 *   gs   = 2688 / amax (1 if amax == 0)            (device scalar, fp32)
 *   s    = e4m3_rn_satfinite((blockmax / 6) * gs)    per 16 elements
 *   q    = e2m1_rne(x * (gs / float(s)))             (0 where s == 0)
 * codes [rows, k/2] uint8 (element 2j in the low nibble), sf [rows, k/16] E4M3.
 * `amax` is a device fp32 scalar (from fgg_amax or supplied by the caller).
 * decode_scale: optional device fp32 scalar that receives g = 1 / gs (the
 * per-tensor decode scale, x ~ e2m1 * e4m3 * g); NULL to skip. */
FGG_API int fgg_nvfp4_quantize(const void* x, int32_t x_dtype, int64_t rows, int32_t k,
                               const float* amax, void* codes, void* sf, float* decode_scale,
                               void* stream);

/* ------------------------------------------------------------------------ */
/* Status                                                                    */
/* ------------------------------------------------------------------------ */

/* Synchronises `stream`, then reads the status word a previous GEMM call left
 * in `workspace` (the NVFP4 or MX workspace).  Returns FGG_OK, FGG_ETIMEOUT
 * (a device wait ran out; the kernel stopped early and its output is
 * incomplete) or FGG_ECUDA. */
FGG_API int fgg_read_device_status(const void* workspace, void* stream);

/* Test hook, no counterpart in the reference: flags applied to every GEMM
 * launch until changed (process-wide).  FGG_DEBUG_NO_LOADS makes the
 * producer arm no pipeline stage and issue no load, so the MMA role's bounded
 * wait on its first stage runs out (after about one second) and the kernel
 * ends early with a non-zero status word: a way to exercise the device error
 * path without a fault.  Returns the previous flags.  0 in normal use. */
#define FGG_DEBUG_NO_LOADS 1
FGG_API int32_t fgg_debug_set_flags(int32_t flags);

#ifdef __cplusplus
}
#endif

#endif /* FGG_API_H */
