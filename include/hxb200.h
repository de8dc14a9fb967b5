/* hxb200.h -- C ABI of the B200 (sm_100a) dispatch library.
 *
 * These are the dispatch-level entry points that replace the Hexagon HMX
 * codegen path of RooflineAI/iree-hexagon-plugins for the dense matmul and
 * attention dispatches. Every pointer argument is a device pointer (CUDA
 * global memory of the current device) unless it says otherwise; `stream` is
 * a cudaStream_t (NULL = legacy default stream). Calls are asynchronous on
 * `stream`; argument errors are reported synchronously through the return
 * status, device-side wait timeouts through hxb_device_status().
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   - the HMX microkernel ABI the compiler emits calls to,
 *     plugins/runtime/hexagon/dsp/ukernel/hmx/api.h:22-67
 *     (acc_clear / pack / mma / acc_read / unpack per 32x32 tile), driven by
 *     the K-loop of plugins/compiler/hexagon/CodeGen/Transforms/
 *     HexagonExpandHmxMatmul.cpp:286-331 -- collapsed here into one call per
 *     linalg.matmul dispatch;
 *   - the decomposed attention dispatches of
 *     examples/attention_layer/attention_layer.mlir:17-111.
 * No torch types appear anywhere in this ABI.
 */
#ifndef HXB200_H_
#define HXB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HXB_ABI_VERSION 1

typedef enum hxb_status_e {
  HXB_OK = 0,
  HXB_STATUS_INVALID_ARGUMENT = 1,
  HXB_STATUS_UNSUPPORTED = 2,
  HXB_STATUS_CUDA_ERROR = 3,
  HXB_STATUS_RESOURCE_EXHAUSTED = 4,
  HXB_STATUS_DEVICE_TIMEOUT = 5,
  HXB_STATUS_UNAVAILABLE = 6,    /* e.g. a driver name no factory provides */
  HXB_STATUS_ALREADY_EXISTS = 7, /* e.g. a factory registered twice */
} hxb_status_t;

typedef enum hxb_dtype_e {
  HXB_DTYPE_F16 = 0,
  HXB_DTYPE_F32 = 1,
  HXB_DTYPE_I8 = 2,
} hxb_dtype_t;

/* Device status bits (hxb_device_status). */
#define HXB_DEVICE_STATUS_TIMEOUT 1

/* ABI version compiled into the library (HXB_ABI_VERSION). */
int hxb_abi_version(void);

/* Text of the last error returned on the calling thread. */
const char* hxb_last_error_message(void);

/* Reads the current device's status word (bits OR-ed in by kernels whose
 * bounded waits gave up) and clears it if `clear` is non-zero. Synchronous. */
hxb_status_t hxb_device_status(int clear, int* out_bits);

/* Self-test of the failure path behind HXB_DEVICE_STATUS_TIMEOUT: launches
 * one CTA whose producer, MMA-issuer and epilogue roles wait, through the
 * same bounded mbarrier wait as every kernel of this library, on a barrier
 * nothing arrives at, with the limit `limit_ns` (at most 1 s) instead of the
 * library's 2 s. The producer has a 4096-byte bulk copy of `src` (device,
 * 16-byte aligned) in flight and the issuer holds TMEM while they wait. The
 * kernel then takes the product failure path -- abort flag, status bit, a
 * bounded wait for the copy, TMEM freed -- and writes 4 int32 to `result`
 * (device): waits that succeeded (0), the abort flag (1), copy intact (1),
 * TMEM freed (1). The status word keeps HXB_DEVICE_STATUS_TIMEOUT until
 * hxb_device_status(1, ...) clears it. The reference has no counterpart (its
 * DSP dispatches report failure through their return code,
 * plugins/runtime/hexagon/dsp/rt/executable_library.h:163-177). */
hxb_status_t hxb_selftest_wait_timeout(uint64_t limit_ns, const void* src,
                                       int32_t* result, void* stream);

/* f16 matmul dispatch: C[M,N] = A[M,K] . B (+ C_init), f32 accumulation.
 *
 * Replaces the HMX lowering of linalg.matmul (f16 x f16 -> f32 init, or f16
 * out), i.e. the per-tile calls iree_hexagon_hmx_pack_f16 /
 * pack_transposed_f16 / mma_f16 / acc_read_f16 / unpack_acc_f16_to_{f32,f16}
 * (plugins/runtime/hexagon/dsp/ukernel/hmx/api.h:22-67) and the DPS init add
 * of the unpack (hmx.c:334-336; HexagonConvertMatmulToHmx.cpp:603-607).
 *
 *   A       f16, row-major [M,K], leading dimension lda (elements)
 *   B       f16, row-major [K,N] (transpose_b = 0) or [N,K] (transpose_b = 1,
 *           the rhs-transposed matmul), leading dimension ldb
 *   C_init  optional (NULL = zeros) addend of C's type and layout
 *   C       row-major [M,N], dtype HXB_DTYPE_F16 or HXB_DTYPE_F32, ldc
 *   workspace / workspace_bytes: device scratch for re-pitching operands
 *           whose row pitch is not a multiple of 16 bytes (TMA requirement);
 *           hxb_matmul_f16_workspace_bytes() tells how much. Pass NULL/0 when
 *           it returns 0.
 * M, N, K >= 1. Returns HXB_STATUS_INVALID_ARGUMENT for bad shapes/strides or
 * a too-small workspace. */
hxb_status_t hxb_matmul_f16(const void* A, int64_t lda, const void* B,
                            int64_t ldb, int transpose_b, const void* C_init,
                            void* C, int64_t ldc, hxb_dtype_t c_dtype,
                            int64_t M, int64_t N, int64_t K, void* workspace,
                            size_t workspace_bytes, void* stream);

/* The tile plan hxb_matmul_f16 uses for a shape on a device with num_sms SMs:
 * the N extent of one output tile (64, 128, 256, or 512 on a CTA pair), the raster group (tile
 * rows swept together for L2 reuse), the K split and the CTA pairing. split_k
 * 1 runs a persistent kernel walking whole tiles; 2, 4 or 8 run one
 * thread-block cluster of that many CTAs per 128-row tile, each on its share
 * of the K-blocks, the partial sums added through distributed shared memory
 * (for shapes whose tiles alone would leave SMs idle). cta_pair 1 gives each
 * SM 128-row tiles; 2 gives a pair of SMs 256-row tiles computed by
 * cta_group::2 MMAs, each SM loading half of the operands (split_k 1 only).
 * Shapes measured by the offline sweep (tile_sweep.py) come from the baked
 * table, the rest from the cost model. This is the B200 counterpart of the
 * reference's HMX tile search, selectHmxTileSizes
 * (plugins/compiler/hexagon/CodeGen/Strategy/Planning/VTCMPlanning.cpp:
 * 186-260). split_k and cta_pair may be NULL. Host only. */
hxb_status_t hxb_plan_matmul_f16(int64_t M, int64_t N, int64_t K, int transpose_b,
                                 int num_sms, int* block_n, int* group_m, int* split_k,
                                 int* cta_pair);

/* hxb_matmul_f16 (no init, no re-pitching) with the tile plan given
 * explicitly instead of planned: the entry the offline tile sweep measures
 * candidates through. block_n in {64, 128, 256}, or 512 with cta_pair 2 (two
 * 256-column MMA chunks per operand stage, one TMEM accumulator); group_m >= 1;
 * split_k in {1, 2, 4, 8} with at least split_k 64-deep K-blocks; cta_pair 1,
 * or 2 with split_k 1 and block_n 128, 256 or 512. */
hxb_status_t hxb_matmul_f16_tiled(const void* A, int64_t lda, const void* B,
                                  int64_t ldb, int transpose_b, void* C,
                                  int64_t ldc, hxb_dtype_t c_dtype, int64_t M,
                                  int64_t N, int64_t K, int block_n, int group_m,
                                  int split_k, int cta_pair, void* stream);

size_t hxb_matmul_f16_workspace_bytes(const void* A, int64_t lda,
                                      const void* B, int64_t ldb,
                                      int transpose_b, int64_t M, int64_t N,
                                      int64_t K);

/* Size of the scratch array built into the library for
 * hxb_matmul_f16_noalloc (bytes, per device). */
#define HXB_NOALLOC_SCRATCH_BYTES (32u << 20)

/* hxb_matmul_f16 for callers that cannot allocate device memory. This entry
 * point has no counterpart in the reference; it exists for callers that hold
 * only the buffers they were handed -- a compiled dispatch function, which
 * gets its bindings and push constants from the runtime and has no allocator,
 * or code recording a CUDA stream capture, where cudaMalloc is not allowed.
 * Same arguments and results as hxb_matmul_f16 minus the workspace: operands
 * whose row pitch breaks the 16-byte TMA rule are re-pitched into a scratch
 * array that lives in the library image, HXB_NOALLOC_SCRATCH_BYTES on every
 * GPU that loads the library, held until the process exits. Operands that
 * need more re-pitch scratch than that are rejected with
 * HXB_STATUS_INVALID_ARGUMENT. The call allocates nothing. Its first call on a
 * device resolves the scratch's device address (make it before any stream
 * capture; hxb_hal_device_create makes it for its device), and again after
 * the device's context was re-created (cudaDeviceReset). `stream` must
 * belong to the current device. All calls on a device share the scratch and
 * leave their data in it, so calls that overlap on the GPU race: order them
 * on one stream. */
hxb_status_t hxb_matmul_f16_noalloc(const void* A, int64_t lda, const void* B,
                                    int64_t ldb, int transpose_b,
                                    const void* C_init, void* C, int64_t ldc,
                                    hxb_dtype_t c_dtype, int64_t M, int64_t N,
                                    int64_t K, void* stream);

/* Weight-quantised matmul dispatch:
 *   C[M,N] f16 = (A[M,K] f16 . W[K,N] int8) * scale[N] f16, f32 accumulation.
 * The reference has no int8 path (ContractionStrategy.cpp:141 restricts HMX to
 * f16); its semantics are those of the linalg the builder emits (sitofp
 * i8->f32, extf scale->f32, mulf, f32 contraction, truncf). int8 -> f16 is
 * exact, so the per-channel scale factors out of the K sum.
 * M >= 1; M <= 16 is routed to the bandwidth-bound GEMV kernel. lda % 8 == 0,
 * ldw % 16 == 0, ldc % 8 == 0 and 16-byte aligned A, W, C, scale. */
hxb_status_t hxb_matmul_w8a16(const void* A, int64_t lda, const void* W,
                              int64_t ldw, const void* scale, void* C,
                              int64_t ldc, int64_t M, int64_t N, int64_t K,
                              void* stream);

/* hxb_matmul_w8a16 with a residual add: C = (A . W) * scale + R, one f16
 * rounding of the f32 result. R has C's layout (leading dimension ldc) and may
 * alias C. Used by the decoder block's output projections (Hugging Face Llama
 * adds the residual after o_proj and down_proj). */
hxb_status_t hxb_matmul_w8a16_residual(const void* A, int64_t lda, const void* W,
                                       int64_t ldw, const void* scale,
                                       const void* R, void* C, int64_t ldc,
                                       int64_t M, int64_t N, int64_t K,
                                       void* stream);

/* Device scratch hxb_matmul_w8a16_streamk needs on the current device (the
 * same for every shape): 4096 bytes of flags, then one 96 KB f32 partial
 * accumulator per SM. */
size_t hxb_matmul_w8a16_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* Schedule of hxb_matmul_w8a16_streamk for M > 16 rows on num_sms SMs, as
 * the dispatch plans it: *grid CTAs; the first *dp_tiles output tiles (128
 * weight columns x 256 activation rows; tile t is row tile t % ceil(M / 256)
 * of column tile t / ceil(M / 256)) are dealt whole, round-robin, and the
 * K-blocks (64 deep) of the others are cut into *grid equal shares
 * (*dp_tiles == number of tiles: data-parallel). When `pieces` is not NULL it
 * receives up to `cap` records of 5 int32 -- CTA, tile, first K-block, end
 * K-block, and the number of other CTAs whose partial sums the piece adds
 * (non-zero only for the piece that finishes a cut tile) -- in each CTA's
 * processing order, the same enumeration the kernel runs; *count (may be
 * NULL) gets the number of records. Host only, no GPU needed. */
hxb_status_t hxb_plan_matmul_w8a16(int64_t M, int64_t N, int64_t K, int num_sms,
                                   int* grid, int* dp_tiles, int32_t* pieces,
                                   int64_t cap, int64_t* count);

/* hxb_matmul_w8a16 (R optional, may be NULL) that may split K across CTAs
 * (stream-K) when whole output tiles would leave SMs idle in the last wave,
 * e.g. the M = 512 projections of the decoder block. Tiles cut between CTAs
 * are summed in a fixed CTA order, so results are deterministic; they may
 * differ from hxb_matmul_w8a16 in the last f32 bit of a sum.
 * `workspace` (16-byte aligned, >= hxb_matmul_w8a16_workspace_bytes) is
 * owned by the caller; its first 4096 bytes must be zero before the first
 * call and every successful call leaves them zero. Calls sharing a workspace
 * must be ordered (one stream). After a call that set hxb_device_status, zero
 * those bytes again. No counterpart in the reference (its HMX path has no
 * int8 weights, ContractionStrategy.cpp:141). */
hxb_status_t hxb_matmul_w8a16_streamk(const void* A, int64_t lda, const void* W,
                                      int64_t ldw, const void* scale,
                                      const void* R, void* C, int64_t ldc,
                                      int64_t M, int64_t N, int64_t K,
                                      void* workspace, size_t workspace_bytes,
                                      void* stream);

/* Fused attention dispatch: O = softmax(scale * Q.K^T [+ causal mask]) . V,
 * f32 softmax statistics, f16 in/out. Replaces the decomposed f32 dispatches
 * of examples/attention_layer/attention_layer.mlir:17-111 (which scale Q and
 * K^T by sqrt(scale) each; the product is the same scale) including its
 * fully-masked-row rule (rows whose scores are all -inf produce 0,
 * :86-103).
 *   Q [BH, Sq, D], K/V [BH, Skv, D], O [BH, Sq, D], all contiguous f16.
 * D must be 64 or 128. causal != 0 masks key j > query i + (Skv - Sq). */
hxb_status_t hxb_attention_f16(const void* Q, const void* K, const void* V,
                               void* O, int64_t BH, int64_t Sq, int64_t Skv,
                               int64_t D, float scale, int causal,
                               void* stream);

/* hxb_attention_f16 on [batch, S, heads * D] matrices: head h of batch b is
 * columns [h*D, (h+1)*D) of rows [b*S, (b+1)*S) of a row-major matrix with
 * leading dimension ld (elements, multiple of 8). Q, K and V may be column
 * blocks of one fused QKV projection output (ld = 3 * heads * D); O is
 * written in the same [batch, S, heads * D] order, the input layout of the
 * output projection. Same semantics and limits as hxb_attention_f16. */
hxb_status_t hxb_attention_f16_bshd(const void* Q, int64_t ldq, const void* K,
                                    int64_t ldk, const void* V, int64_t ldv,
                                    void* O, int64_t ldo, int64_t batch,
                                    int64_t heads, int64_t Sq, int64_t Skv,
                                    int64_t D, float scale, int causal,
                                    void* stream);

/* Output layouts of hxb_attention_gqa_f16. */
#define HXB_ATTN_OUT_BHSD 0 /* [batch, q_heads, q_len, D] */
#define HXB_ATTN_OUT_BSHD 1 /* [batch, q_len, q_heads, D] */

/* Grouped-query attention over the first kv_len rows of a KV cache, the
 * SlicedCacheAttention of integration_tests/models/micro/
 * attention-cache-slice-f16/model.py:17-31 (SmolLM2's attention against its
 * static cache) and the grouped_query_attention of the KV-cache LMs
 * (integration_tests/models/kv_cache.py:46-86): query head h reads KV head
 * h / (q_heads / kv_heads).
 *   Q    [batch, q_heads, q_len, D] contiguous f16
 *   K, V [batch, kv_heads, kv_rows, D] contiguous f16; rows [0, kv_len)
 *        of each head are attended (kv_len <= kv_rows)
 *   O    out_layout HXB_ATTN_OUT_BHSD or HXB_ATTN_OUT_BSHD (the models'
 *        permute(0, 3, 1, 2, 4) output)
 * q_heads must be a multiple of kv_heads; D 64 or 128; scale > 0 (the models
 * use D^-0.5). causal != 0 masks key j > q_pos0 + i for query i, q_pos0
 * being the cache position of the first query: kv_len - q_len when the
 * queries are the last cached rows (decode, chunked prefill), 0 for a
 * padded prefill whose keys past the last real token are cut by kv_len.
 * Rows that see no key are 0. The query heads of one group share one pass
 * over their KV head's keys.
 * When the query blocks alone would not fill the SMs (decode: a handful of
 * rows per KV head against a long cache) the keys are split across CTAs and
 * the partial results merged by a second kernel; that needs `workspace` of
 * hxb_attention_gqa_workspace_bytes(...) bytes (16-byte aligned, no
 * initial contents). A null or smaller workspace runs without the split.
 * Calls sharing a workspace must be ordered (one stream). */
hxb_status_t hxb_attention_gqa_f16(const void* Q, const void* K, const void* V,
                                   void* O, int64_t batch, int64_t q_heads,
                                   int64_t kv_heads, int64_t q_len,
                                   int64_t q_pos0, int64_t kv_len,
                                   int64_t kv_rows, int64_t D, float scale,
                                   int causal, int out_layout, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Workspace hxb_attention_gqa_f16 uses for its key split on the current
 * device; 0 when that shape runs without a split (or is invalid). */
size_t hxb_attention_gqa_workspace_bytes(int64_t batch, int64_t q_heads,
                                         int64_t kv_heads, int64_t q_len,
                                         int64_t kv_len, int64_t D);

/* ---- N-sharded f16 matmul across GPUs --------
 * The reference has no collectives (plugins/runtime/hexagon/channel.c:55-56
 * returns IREE_STATUS_UNIMPLEMENTED); these entries serve the multi-GPU split
 * of one large matmul along N, each rank computing C[:, its columns]. */

/* f16 matmul whose epilogue also writes every output tile into the other
 * ranks' copies of C over NVLink: an all-gather fused into the GEMM.
 *   C         this rank's column block of its own full [M, ldc] output
 *             (i.e. full_output + column offset of the shard)
 *   replicas  nreplicas (0..7) peer pointers to the same column offset in
 *             the other ranks' full outputs (peer memory, e.g. CUDA IPC)
 * A is [M, K] (lda), B the rank's shard [K, N] or [N, K] (ldb), both with
 * 16-byte aligned rows. The caller orders this call after the peers stopped
 * reading their outputs and synchronises the ranks after it (e.g. a
 * stream-ordered collective) before reading the gathered C. */
hxb_status_t hxb_matmul_f16_allgather(const void* A, int64_t lda, const void* B,
                                      int64_t ldb, int transpose_b, void* C,
                                      void* const* replicas, int nreplicas,
                                      int64_t ldc, int64_t M, int64_t N,
                                      int64_t K, void* stream);

/* int8-weight matmul of one column shard whose output is also written into
 * the other ranks' copies of C over NVLink: the all-gather of the N-split of
 * BASELINE configuration 2 (W [K, N_total] split into column shards of a
 * multiple of 8 columns). Same arguments as hxb_matmul_w8a16_streamk for the
 * shard (W, scale and N are the shard's; C and ldc as in
 * hxb_matmul_f16_allgather: this rank's column block of its full [M, ldc]
 * output) plus nreplicas (0..7) 16-byte aligned peer pointers to the same
 * column offset in the other ranks' outputs. For M > 16 the tcgen05 GEMM's
 * epilogue stores every staged output tile to the replicas as well; for
 * M <= 16 the GEMV's few output rows are copied to them by one small kernel
 * after it. workspace may be NULL (no stream-K). The caller orders the call
 * after the peers stopped reading their outputs and synchronises the ranks
 * after it. No counterpart in the reference (no int8 path, no
 * collectives: plugins/runtime/hexagon/channel.c:55-56). */
hxb_status_t hxb_matmul_w8a16_allgather(const void* A, int64_t lda, const void* W,
                                        int64_t ldw, const void* scale, void* C,
                                        void* const* replicas, int nreplicas,
                                        int64_t ldc, int64_t M, int64_t N, int64_t K,
                                        void* workspace, size_t workspace_bytes,
                                        void* stream);

/* CUDA IPC for the replicas of hxb_matmul_f16_allgather. get_handle fills
 * HXB_IPC_HANDLE_BYTES bytes naming the allocation that holds `ptr` and the
 * byte offset of `ptr` inside it; open maps a peer's allocation into the
 * CURRENT device's context with peer access enabled (so kernels on this
 * device can store into it) and returns the pointer at `offset`; close
 * unmaps it. */
#define HXB_IPC_HANDLE_BYTES 64
hxb_status_t hxb_ipc_get_handle(const void* ptr, void* handle, int64_t* offset);
hxb_status_t hxb_ipc_open(const void* handle, int64_t offset, void** ptr);
hxb_status_t hxb_ipc_close(void* ptr, int64_t offset);

/* Stream-ordered barrier of `world` ranks (one GPU each) through peer
 * memory, for ordering the fused all-gather steps without a collective
 * library call: flags[i] is rank i's array of `world` uint32 flags (this
 * rank's own array at index `rank`, the others mapped with hxb_ipc_open;
 * zero-initialised, 4-byte aligned). Rank r stores `epoch` into every peer's
 * flag r (release, system scope) and waits until every peer's flag in its own
 * array reached `epoch` (acquire). Every rank passes the same increasing
 * epoch (> 0) to its k-th barrier. The wait is bounded by the library's
 * wait limit; a wait that runs out sets HXB_DEVICE_STATUS_TIMEOUT. No
 * counterpart in the reference (no collectives, channel.c:55-56). */
hxb_status_t hxb_peer_barrier(void* const* flags, int world, int rank, uint32_t epoch,
                              void* stream);

/* dst[m, g*n + j] = src[g, m, j]: the [G, M, n] result of an NCCL all-gather
 * of column shards laid out as the [M, G*n] matrix (row pitch ldd).
 * n % 8 == 0, 16-byte aligned buffers. */
hxb_status_t hxb_gather_column_blocks_f16(const void* src, void* dst, int64_t G,
                                          int64_t M, int64_t n, int64_t ldd,
                                          void* stream);

/* ---- Llama-style decoder block ----------------
 * The reference has no decoder kernels of its own; its decoder models are
 * Hugging Face Llama checkpoints run through torch
 * (integration_tests/models/meta-llama/Llama-3.2-1B-Instruct/model.py). The
 * entries below follow the arithmetic of those modules on f16 activations. */

/* y = f16(x * rsqrt(mean(x^2) + eps)) * gamma per row (LlamaRMSNorm:
 * f32 statistics, f16 result times the f16 weight). cols % 8 == 0. */
hxb_status_t hxb_rmsnorm_f16(const void* x, int64_t ldx, const void* gamma,
                             void* y, int64_t ldy, int64_t rows, int64_t cols,
                             float eps, void* stream);

/* In-place rotary embedding of the first `heads` heads (head_dim 128) of every
 * row: pairs (i, i + 64) rotate by (pos0 + row % seq) * theta^(-2i/128)
 * (Llama rotate_half convention). For a fused QKV row pass 2 * n_heads to
 * rotate q and k together. */
hxb_status_t hxb_rope_f16(void* x, int64_t ldx, int64_t rows, int64_t heads,
                          int64_t head_dim, int64_t seq, int64_t pos0,
                          float theta, void* stream);

/* a[r, j] = silu(gu[r, j]) * gu[r, ffn + j] (LlamaMLP: gate columns, then up
 * columns, of one fused gate/up projection output). ffn % 8 == 0. */
hxb_status_t hxb_swiglu_f16(const void* gu, int64_t ldgu, void* a, int64_t lda,
                            int64_t rows, int64_t ffn, void* stream);

/* Weights of one decoder block. int8 matrices are [in, out] row-major with an
 * f16 per-output-column scale; w_gate_up holds the gate columns then the up
 * columns ([hidden, 2 * ffn]). Norm weights are f16 [hidden]. */
typedef struct hxb_decoder_w8_s {
  int64_t hidden, heads, head_dim, ffn;
  float rms_eps, rope_theta;
  const void* attn_norm;
  const void* w_qkv;      /* [hidden, 3 * hidden]: q, k, v column blocks */
  const void* s_qkv;
  const void* w_o;        /* [hidden, hidden] */
  const void* s_o;
  const void* ffn_norm;
  const void* w_gate_up;  /* [hidden, 2 * ffn] */
  const void* s_gate_up;
  const void* w_down;     /* [ffn, hidden] */
  const void* s_down;
} hxb_decoder_w8_t;

/* Device workspace hxb_decoder_block_w8a16 needs for batch * seq rows
 * (0 if the weights description is invalid). */
size_t hxb_decoder_block_workspace_bytes(const hxb_decoder_w8_t* w,
                                         int64_t batch, int64_t seq);

/* out = decoder_block(x): x, out [batch * seq, hidden] f16 row-major,
 * causal self-attention over each batch's seq rows at positions pos0 .. The
 * block runs as a sequence of dispatches on `stream` (RMSNorm, QKV W8 GEMM,
 * RoPE, attention, O W8 GEMM + residual, RMSNorm, gate/up W8 GEMM, SwiGLU,
 * down W8 GEMM + residual). */
hxb_status_t hxb_decoder_block_w8a16(const hxb_decoder_w8_t* w, const void* x,
                                     void* out, int64_t batch, int64_t seq,
                                     int64_t pos0, void* workspace,
                                     size_t workspace_bytes, void* stream);

/* KV-cache update (SliceUpdateKvCache.update,
 * integration_tests/models/kv_cache.py:101-112):
 *   k_cache[b, h, begin + t, :] = k_src[b * n + t, h*D : (h+1)*D]
 *   v_cache[b, h, begin + t, :] = v_src[b * n + t, h*D : (h+1)*D]
 * for t < n. Sources are row-major [batch * n, ld_src] f16 (e.g. the K and V
 * column blocks of a fused QKV output, ld_src = 3 * hidden); caches are
 * [batch, kv_heads, cache_rows, D] f16. begin + n <= cache_rows. */
hxb_status_t hxb_kv_cache_write_f16(const void* k_src, const void* v_src,
                                    int64_t ld_src, void* k_cache, void* v_cache,
                                    int64_t batch, int64_t kv_heads, int64_t n,
                                    int64_t begin, int64_t cache_rows,
                                    int64_t head_dim, void* stream);

/* Device workspace hxb_decoder_block_w8a16_cached needs for batch * seq new
 * rows (0 if the weights description is invalid). */
size_t hxb_decoder_block_cached_workspace_bytes(const hxb_decoder_w8_t* w,
                                                int64_t batch, int64_t seq);

/* The decoder block against a KV cache, the prefill / decode steps of the
 * reference's KV-cache LMs (integration_tests/models/kv_cache.py:145-186):
 * the seq new rows of each batch are at positions pos0 .. pos0 + seq - 1;
 * their rotated K and their V are written into k_cache / v_cache
 * ([batch, heads, cache_rows, head_dim] f16) at rows pos0 .., and attention
 * reads keys [0, pos0 + seq) from the caches, causally. pos0 = 0 with the
 * whole prompt is the prefill (same result as hxb_decoder_block_w8a16);
 * seq = 1 at pos0 = the tokens so far is one decode step. Short steps split
 * the keys across SMs. */
hxb_status_t hxb_decoder_block_w8a16_cached(const hxb_decoder_w8_t* w,
                                            const void* x, void* out,
                                            int64_t batch, int64_t seq,
                                            int64_t pos0, void* k_cache,
                                            void* v_cache, int64_t cache_rows,
                                            void* workspace,
                                            size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HXB200_H_ */
