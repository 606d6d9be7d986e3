/*
 * nvfp4_qsa.h -- C ABI of the B200 (sm_100a) NVFP4 paged KV-cache writer and
 * QSA sparse decode attention.
 *
 * Every entry point takes plain device pointers, element counts and strides,
 * and a cudaStream_t passed as `void*` (NULL = legacy default stream).  No
 * entry point allocates, synchronizes the stream, or reads device memory from
 * the host, so every launch is legal inside CUDA graph capture.  All entry
 * points return an nvqsa_status code; NVQSA_OK is 0.
 *
 * Cache layout (reference python/nvfp4_qsa/cache.py:20-24): one uint8 tensor
 * [blocks, kv_heads, page, 2*(head_dim/2 + head_dim/16)] viewed as four
 * regions, each indexed [block, token_in_page, kv_head, byte]:
 *   key_data   head_dim/2  bytes  E2M1 nibbles, low nibble = element 2j
 *   key_scale  head_dim/16 bytes  E4M3 group scale, one per 16 elements
 *   value_data head_dim/2  bytes
 *   value_scale head_dim/16 bytes
 * The ABI takes each region's base pointer and its (block, token, head) byte
 * strides, so any layout whose innermost byte run is contiguous is accepted.
 */
#ifndef NVFP4_QSA_H_
#define NVFP4_QSA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum nvqsa_status {
  NVQSA_OK = 0,
  NVQSA_ERR_NULL_POINTER = 1,   /* a required pointer is NULL */
  NVQSA_ERR_BAD_SHAPE = 2,      /* negative / inconsistent sizes */
  NVQSA_ERR_HEAD_DIM = 3,       /* head_dim not supported by this build */
  NVQSA_ERR_MISALIGNED = 4,     /* pointer or stride breaks the alignment contract */
  NVQSA_ERR_WORKSPACE = 5,      /* workspace missing or smaller than required */
  NVQSA_ERR_UNSUPPORTED = 6,    /* head grouping / block size outside this build */
  NVQSA_ERR_LAUNCH = 7,         /* the CUDA launch itself failed */
  NVQSA_ERR_CUDA = 8,           /* a CUDA runtime query failed */
  NVQSA_ERR_SCRATCH_LIMIT = 9   /* problem needs more scratch than the built-in buffer holds */
};

/* Human-readable text for a status code (static storage). */
const char* nvqsa_status_string(int status);

/* ABI revision of this library; bumped when a signature changes. */
int nvqsa_abi_version(void);

/*
 * Device error flags raised by the kernels on the current device (bit 0: a
 * bounded wait on a shared-memory barrier ran out, the affected CTA skipped
 * its output; bit 1: a split-KV peer's slot did not arrive within 2 s; bit 2:
 * a bounded wait of nvqsa_kv_proj_write_cache ran out).  Kernels never trap; this synchronous query (it copies one
 * word from the device) is for tests and diagnostics.  clear != 0 resets the
 * flags after reading.  No counterpart in the reference.
 */
int nvqsa_read_error_flags(uint32_t* flags, int clear);

/*
 * Quantize BF16 K and V rows to NVFP4 and scatter them into the paged cache in
 * ONE launch.
 *
 * Replaces qsa_write_cache_nvfp4 (reference python/nvfp4_qsa/kernels.py:152-165),
 * which runs _write_one (kernels.py:118-149) twice.  Per (token t, kv head h):
 * slot = slot_mapping[t]; the token is skipped when slot < 0 or
 * slot / page_size >= num_blocks (kernels.py:71-77).  Each group of 16
 * values gets scale = e4m3_rn(min(g * amax / 6, 448)) and nibbles
 * e2m1_rn(clamp(x * g / max(scale, 1e-30), -6, 6)); the bytes equal the
 * reference codec oracle (python/nvfp4_qsa/oracle.py:47-69) for every finite
 * input, including groups whose scale rounds to zero.
 *
 * key, value : bf16 [num_tokens, kv_heads, head_dim], element strides given,
 *              innermost stride 1.
 * *_data / *_scale : cache regions, byte strides (block, token, head).
 * slot_mapping : int64 [num_tokens].
 * head_dim : 64, 128, 256 or 512.
 */
int nvqsa_write_cache(
    const void* key, int64_t key_stride_token, int64_t key_stride_head,
    const void* value, int64_t value_stride_token, int64_t value_stride_head,
    void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    const int64_t* slot_mapping, int64_t num_tokens, int32_t kv_heads, int32_t head_dim,
    int64_t num_blocks, int64_t page_size,
    float key_global_scale, float value_global_scale, void* stream);

/*
 * nvqsa_write_cache with the K rows first passed through the caller's k-norm
 * and rotary embedding, in the same launch: K is read once from the QKV
 * projection output and never written back as bf16 unless key_out asks for it.
 *
 * Replaces, at the reference's call site (integration/snapshot/qsa.py:618-667:
 * qkv_proj -> k_norm (vLLM GemmaRMSNorm) -> rotary_emb -> qsa_write_cache_nvfp4),
 * the k_norm and rotary steps for K plus the writer.  Per (token t, kv head h):
 *   norm (norm_weight != NULL):
 *     ss = sum_d x[d]^2 in fp32, x[d] bf16: 32 partial sums, partial l over
 *          d in [l*E, l*E+E) (E = head_dim/32) as (FMA-sum of the squares at
 *          even d, in order) + (FMA-sum of those at odd d, in order); the 32
 *          partials added pairwise at distances 16, 8, 4, 2, 1
 *     r  = 1 / sqrt(ss / head_dim + eps)             (IEEE sqrt and divide)
 *     y[d] = bf16_rn((x[d] * r) * (norm_weight[d] + norm_weight_offset))
 *          (norm_weight_offset = 1 for GemmaRMSNorm, 0 for a plain RMSNorm
 *          with fp32 weights); without a norm, y = x.
 *   rotation (rotary_dim > 0): c, s = cos_sin_cache[positions[t]] halves
 *     (bf16 [max_position, cos_sin_stride], cos in [0, rotary_dim/2), sin in
 *     [rotary_dim/2, rotary_dim)); NeoX pairs (y[i], y[i + rotary_dim/2]),
 *     GPT-J pairs (y[2i], y[2i+1]):
 *       o1 = bf16(bf16(x1 c) - bf16(x2 s)), o2 = bf16(bf16(x2 c) + bf16(x1 s))
 *     -- vLLM's native rotary embedding in bf16 arithmetic, bit for bit.
 *     Elements at or past rotary_dim pass through.
 *   then K (rotated) and V (unchanged) are encoded and scattered exactly as
 *   nvqsa_write_cache does; key_out (optional, bf16 [num_tokens, kv_heads,
 *   head_dim] with element strides, base and strides aligned to
 *   min(head_dim/16, 16) bytes, else NVQSA_ERR_MISALIGNED) receives the
 *   rotated K of every token whose position is valid, whatever its slot.
 * A token whose position is outside [0, max_position) is skipped entirely
 * (no cache bytes, no key_out row).  rotary_dim must be a multiple of
 * head_dim/16 and at most head_dim (NVQSA_ERR_BAD_SHAPE); the table's base
 * and row stride must be aligned to head_dim/16 bytes for NeoX, head_dim/32
 * for GPT-J (NVQSA_ERR_MISALIGNED; a contiguous table is); rotary_dim = 0 and
 * norm_weight = NULL give the plain writer.  eps must be finite and >= 0.
 * No counterpart entry in the reference (its writer takes K after the norm
 * and rotation).
 */
int nvqsa_norm_rope_write_cache(
    const void* key, int64_t key_stride_token, int64_t key_stride_head,
    const void* value, int64_t value_stride_token, int64_t value_stride_head,
    void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    const int64_t* slot_mapping, int64_t num_tokens, int32_t kv_heads, int32_t head_dim,
    int64_t num_blocks, int64_t page_size, float key_global_scale, float value_global_scale,
    const float* norm_weight, float norm_weight_offset, float eps,
    const int64_t* positions, const void* cos_sin_cache, int64_t cos_sin_stride, int64_t max_position,
    int32_t rotary_dim, int32_t is_neox_style,
    void* key_out, int64_t key_out_stride_token, int64_t key_out_stride_head, void* stream);

/*
 * The K and V columns of the attention layer's QKV projection, computed and
 * written to the NVFP4 cache in ONE launch (tensor-core GEMM whose epilogue is
 * nvqsa_norm_rope_write_cache): the bf16 K and V never go through HBM.
 *
 * Replaces, at the reference's call site (integration/snapshot/qsa.py:658-667
 * -> :618-640: qkv_proj -> split -> k_norm -> rotary_emb ->
 * qsa_write_cache_nvfp4), the K/V part of the projection plus the norm,
 * rotation and writer.  For token t and kv head h:
 *   K[t, h, :] = bf16_rn(sum_c hidden[t, c] * key_weight[h*256 + d, c]),
 *   V likewise with value_weight (fp32 accumulation; the order of the sum is
 *   the tensor cores', so a value can differ by one bf16 ulp from another
 *   GEMM's), then K goes through the norm and rotation and both are encoded
 *   and scattered exactly as nvqsa_norm_rope_write_cache does with these K and
 *   V (same skip rules for positions and slots, same bytes).
 * hidden    : bf16 [num_tokens, hidden_size], row stride hidden_stride_token
 *             elements; key_weight / value_weight: bf16 [kv_heads*256,
 *             hidden_size] (the K and V row blocks of the QKV weight), row
 *             stride weight_stride_row.  Bases 16-byte aligned, row strides
 *             multiples of 8 elements (NVQSA_ERR_MISALIGNED).
 * head_dim  : 256 only (NVQSA_ERR_HEAD_DIM).
 * cache     : the four regions must be views of one [blocks, kv_heads, page,
 *             288]-style record storage with shared strides (the reference's
 *             and vLLM's layout) and 16-byte aligned strides and region
 *             bases, else NVQSA_ERR_MISALIGNED.
 * rotation  : rotary_dim a multiple of 32 (NeoX) or 16 (GPT-J), at most 256;
 *             the cos/sin table's base and row stride 16-byte aligned.
 * norm_weight (fp32 [256], 16-byte aligned) or NULL; eps as the fused writer.
 * key_out   : optional bf16 [num_tokens, kv_heads, 256] rotated K (rows of
 *             tokens with a valid position), value_out: optional bf16 V
 *             projection (every token); bases and strides 16-byte aligned.
 * A wait of the kernel that runs out sets bit 2 of nvqsa_read_error_flags.
 * No counterpart entry in the reference (its projection is vLLM's GEMM).
 */
int nvqsa_kv_proj_write_cache(
    const void* hidden, int64_t hidden_stride_token, int64_t num_tokens, int32_t hidden_size,
    const void* key_weight, const void* value_weight, int64_t weight_stride_row,
    void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    const int64_t* slot_mapping, int32_t kv_heads, int32_t head_dim,
    int64_t num_blocks, int64_t page_size, float key_global_scale, float value_global_scale,
    const float* norm_weight, float norm_weight_offset, float eps,
    const int64_t* positions, const void* cos_sin_cache, int64_t cos_sin_stride, int64_t max_position,
    int32_t rotary_dim, int32_t is_neox_style,
    void* key_out, int64_t key_out_stride_token, int64_t key_out_stride_head,
    void* value_out, int64_t value_out_stride_token, int64_t value_out_stride_head, void* stream);

/*
 * Bytes of workspace nvqsa_sparse_attention needs for this problem on the
 * current device (0 when the problem runs without a split-KV merge).
 */
int nvqsa_sparse_attention_workspace_size(
    int64_t rows, int32_t query_heads, int32_t kv_heads, int32_t head_dim,
    int64_t topk, size_t* workspace_bytes);

/*
 * QSA sparse paged decode attention over an NVFP4 cache.
 *
 * Replaces qsa_sparse_paged_attention_nvfp4 (reference
 * python/nvfp4_qsa/kernels.py:348-403, kernel :168-345).  For query row r and
 * kv head h, the query heads h*G .. h*G+G-1 (G = query_heads / kv_heads)
 * attend to the selected tokens logical_indices[r, 0:topk] of request
 * token_to_request[r]: token i lives in physical block
 * block_table[req, i / page_size] at offset i % page_size.  A selection is
 * masked when req is outside [0, num_requests), the index is negative, its
 * page is >= table_width, or the physical block is outside [0, num_blocks)
 * (kernels.py:241-257); duplicates count once per occurrence; a row with no
 * valid selection produces zeros (kernels.py:333-337).  Scores use
 * head_dim^-0.5 / key_global_scale, the output is divided by
 * value_global_scale and stored as bf16.
 *
 * query, output : bf16 [rows, query_heads, head_dim], element strides given,
 *                 innermost stride 1.  Only rows [0, rows) are written.
 * logical_indices : int32 [rows, topk] contiguous.
 * block_table     : int32 [num_requests, table_width] contiguous.
 * token_to_request: int32 [rows].
 * Cache region pointers and byte strides must be 16-byte aligned.
 * head_dim must be 256, G must be 1..16, and both global scales must be
 * finite and positive (NVQSA_ERR_BAD_SHAPE otherwise).
 * workspace : device memory of at least nvqsa_sparse_attention_workspace_size
 *             bytes (may be NULL when that size is 0); contents need no
 *             initialisation and are dead after the call.  It holds the
 *             split-KV partials and one arrival counter per (row, kv head),
 *             which the call zeroes on `stream` (a memset node when captured)
 *             before its one kernel launch; the last CTA of each (row, kv
 *             head) merges that unit's partials.
 */
int nvqsa_sparse_attention(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Grouped variant for multi-token-prediction (MTP) decode batches, where the
 * draft rows of a sequence attend to one shared selection list: rows
 * [g * rows_per_group, (g + 1) * rows_per_group) form group g.  Same
 * arguments, masking and result as nvqsa_sparse_attention (the reference
 * interface it extends is qsa_sparse_paged_attention_nvfp4,
 * python/nvfp4_qsa/kernels.py:348-403); rows_per_group is a hint only.  When
 * rows_per_group * G <= 48, rows_per_group is 2..4 and the cache is the
 * canonical [blocks, kv_heads, page, 288] storage, each selected record is
 * gathered and dequantised once per group instead of once per row; every CTA
 * verifies on the device that the group's rows have the same request and the
 * same selections for its share of the index positions, and processes a
 * group that does not share row by row.  Otherwise (or with rows_per_group
 * 1) the call is nvqsa_sparse_attention.  The grouped kernel needs no
 * workspace; pass the one nvqsa_sparse_attention_workspace_size gives.
 * rows_per_group outside 1..4 -> NVQSA_ERR_BAD_SHAPE.
 */
int nvqsa_sparse_attention_grouped(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim, int32_t rows_per_group,
    void* workspace, size_t workspace_bytes, void* stream);

/*
 * FP8 sibling reader: the same sparse paged decode attention over float8_e4m3
 * K and V caches (one byte per element) instead of NVFP4 records.  Replaces
 * the reference's qsa_sparse_paged_attention_fp8 (src/qsa_fp8_harness.py:211-325,
 * kernel :42-208; called from integration/snapshot/qsa.py:328-350).
 *
 * key_cache, value_cache : float8_e4m3fn [num_blocks, page_size, kv_heads,
 *                          head_dim] with byte strides (block, token, head),
 *                          innermost stride 1; 16-byte aligned rows and strides.
 * k_scale multiplies the scores (with head_dim^-0.5), v_scale the normalised
 * output, both per-tensor, finite and positive.  Masking, split-KV and the
 * workspace as for nvqsa_sparse_attention (size from
 * nvqsa_sparse_attention_workspace_size with the same rows, heads and topk).
 */
int nvqsa_sparse_attention_fp8(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_cache, int64_t kc_stride_block, int64_t kc_stride_token, int64_t kc_stride_head,
    const void* value_cache, int64_t vc_stride_block, int64_t vc_stride_token, int64_t vc_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads, float k_scale, float v_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes, void* stream);

/*
 * BF16 sibling reader: the same sparse paged decode attention over the bf16
 * main cache (no quantisation).  Replaces vLLM's qsa_sparse_paged_attention
 * that the reference calls in the third branch of forward_qsa
 * (integration/snapshot/qsa.py:352-366); its arithmetic is the FP8 harness
 * kernel's without the dequantisation (src/qsa_fp8_harness.py:42-208, scale
 * head_dim^-0.5, P cast to bf16 before P V).
 *
 * key_cache, value_cache : bf16 [num_blocks, page_size, kv_heads, head_dim]
 *                          with BYTE strides (block, token, head), innermost
 *                          stride 1 element; 16-byte aligned rows and strides
 *                          (vLLM's views of a [blocks, kv_heads, page, 2*256]
 *                          bf16 cache qualify).
 * Masking, output and split-KV rules as nvqsa_sparse_attention; the workspace
 * size comes from nvqsa_sparse_attention_bf16_workspace_size.
 */
int nvqsa_sparse_attention_bf16(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_cache, int64_t kc_stride_block, int64_t kc_stride_token, int64_t kc_stride_head,
    const void* value_cache, int64_t vc_stride_block, int64_t vc_stride_token, int64_t vc_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes nvqsa_sparse_attention_bf16 needs for this shape on the current device. */
int nvqsa_sparse_attention_bf16_workspace_size(int64_t rows, int32_t query_heads, int32_t kv_heads, int32_t head_dim,
                                               int64_t topk, size_t* workspace_bytes);

/*
 * Partial (un-merged) variant for split-KV across devices: writes, for every
 * (row, query head), the softmax-normalized output of the selections this
 * device holds, already divided by value_global_scale, and its base-2
 * log-sum-exp (max + log2(sum), or -inf when the device holds none of the
 * row's selections).  Selections whose block-table entry is outside
 * [0, num_blocks) are masked, so each device passes a block table that maps
 * only the pages it owns.  Partial format follows the reference's split-K
 * sibling (src/qsa_fp8_harness.py:183-208).
 *
 * partial_out : fp32 [rows, query_heads, head_dim] contiguous.
 * partial_lse : fp32 [rows, query_heads] contiguous.
 * Other arguments as nvqsa_sparse_attention; workspace sized by
 * nvqsa_sparse_attention_workspace_size.
 */
int nvqsa_sparse_attention_partial(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    float* partial_out, float* partial_lse,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Split-KV decode of one sequence across GPUs, the exchange fused into the
 * reader kernel: each rank runs this call on its own cache pages (its block
 * table holds -1 on pages other ranks own, so its share of the selections is
 * implicit).  The CTA that finishes this rank's merged (O, lse) of a (row,
 * kv head) stores it into slot `rank` of every rank's exchange buffer over
 * NVLink, raises that rank's flag (release), waits for the flags of all
 * other ranks (acquire; bounded at 2 s, after which bit 1 of the device error
 * flags is raised and the output is left unwritten) and merges the `world`
 * slots into `output` (bf16).  Every rank gets the full result.  This
 * replaces the reference's split-K merge (src/qsa_fp8_harness.py:308-321)
 * done after an all_gather; there is no reference counterpart for the
 * peer-memory exchange itself.
 *
 * exchange : [world] pointers, rank r's exchange buffer as mapped in this
 *            process (own buffer included; peers via nvqsa_ipc_open_handle),
 *            each nvqsa_split_kv_exchange_bytes(rows, ...) bytes, allocated
 *            by nvqsa_exchange_alloc (zeroed).  The same `rows` on every call.
 * parity   : 0 or 1, alternating from call to call on this exchange buffer
 *            (every rank the same sequence), so a fast rank's next call never
 *            meets flags of the previous one.
 * All ranks must make the same calls in the same order; calls are not
 * capture-safe across ranks (eager use).
 */
int nvqsa_split_kv_exchange_bytes(int64_t rows, int32_t query_heads, int32_t kv_heads, int32_t world,
                                  size_t* bytes);
int nvqsa_exchange_alloc(size_t bytes, void** ptr);
int nvqsa_exchange_free(void* ptr);
/* CUDA IPC handle (64 bytes) of an exchange buffer, and mapping a peer's handle into this process. */
int nvqsa_ipc_get_handle(const void* ptr, void* handle);
int nvqsa_ipc_open_handle(const void* handle, void** ptr);
int nvqsa_ipc_close_handle(void* ptr);
int nvqsa_sparse_attention_split_kv(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim,
    void* workspace, size_t workspace_bytes,
    void* const* exchange, int32_t world, int32_t rank, int32_t parity, void* stream);

/*
 * Log-sum-exp merge of `splits` partials into the bf16 output: for each
 * (row, head), out = sum_s 2^(lse_s - M) * O_s / sum_s 2^(lse_s - M) with
 * M = max_s lse_s; rows whose partials are all -inf become zeros.  The
 * merge step of the reference's split-K sibling (src/qsa_fp8_harness.py:308-321).
 *
 * partial_out : fp32 [splits, rows, query_heads, head_dim] contiguous.
 * partial_lse : fp32 [splits, rows, query_heads] contiguous.
 * output      : bf16 [rows, query_heads, head_dim], innermost stride 1.
 */
int nvqsa_merge_partials(
    const float* partial_out, const float* partial_lse, int32_t splits,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim, void* stream);

/*
 * nvqsa_merge_partials with the splits at any distance: split s starts at
 * partial_out + s * out_split_stride and partial_lse + s * lse_split_stride
 * (in floats), each split dense [rows, query_heads, head_dim] / [rows,
 * query_heads].  Used by the split-KV decode across GPUs, whose all_gather
 * leaves every rank's outputs and lse packed in one buffer.  No reference
 * counterpart of its own: the reference's split-K merge is the vLLM kernel
 * called at src/qsa_fp8_harness.py:308-321.
 * out_split_stride must be a multiple of 4 floats.
 */
int nvqsa_merge_partials_strided(
    const float* partial_out, int64_t out_split_stride,
    const float* partial_lse, int64_t lse_split_stride, int32_t splits,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim, void* stream);

/*
 * Flat NVFP4 codec on device rows (the GPU form of the reference codec
 * encode(), python/nvfp4_qsa/oracle.py:47-69).
 *
 * x           : fp32 [m, n] contiguous, n % block_size == 0, block_size even.
 * global_scale: device pointer to one fp32.
 * nibbles     : uint8 [m, n] (may be NULL), packed : uint8 [m, n/2],
 * scales      : uint8 [m, n/block_size].
 * counts      : device int64[2], accumulated (caller zeroes): [0] = elements
 *               with |x * g / scale| > 6, [1] = groups whose unrounded scale
 *               is >= 448 - 1e-3 (may be NULL).
 */
int nvqsa_encode_rows(
    const float* x, int64_t m, int64_t n, int32_t block_size, const float* global_scale,
    uint8_t* nibbles, uint8_t* packed, uint8_t* scales, int64_t* counts, void* stream);

/*
 * Inverse of nvqsa_encode_rows (reference oracle.py:72-85):
 * out[i, j] = e2m1(nibble) * (e4m3(scale) / g), fp32 [m, n] contiguous.
 */
int nvqsa_decode_rows(
    const uint8_t* packed, const uint8_t* scales, int64_t m, int64_t n, int32_t block_size,
    const float* global_scale, float* out, void* stream);


/*
 * QSA indexer top-k: the selection that fills the reader's logical_indices.
 * The reference's QSA layer hands its (un-vendored) indexer the buffer
 * topk_indices_buffer[:num_tokens], int32 [num_tokens, output_width], and
 * requires that shape back (integration/snapshot/qsa.py:537-545, :605-616).
 * For each row, among scores[row, 0 .. lengths[row]) (all `context` when
 * lengths is NULL), the indices of the k largest, ascending; ties at the k-th
 * value go to the lowest indices; NaN ranks above every number; a row with
 * fewer than k valid positions gets 0 .. len - 1 followed by -1.
 *
 * scores : fp32 [rows, context], row stride score_stride_row >= context elements
 * out    : int32 [rows, k], row stride out_stride_row >= k elements
 */
int nvqsa_topk_indices(const float* scores, int64_t score_stride_row, const int32_t* lengths, int64_t rows,
                       int64_t context, int32_t k, int32_t* out, int64_t out_stride_row, void* stream);

/*
 * Measurement aid, no counterpart in the reference: install (stamps != NULL)
 * or remove (NULL) a device buffer of uint64 %globaltimer stamps for the
 * current device.  While installed, every reader launch on that device
 * writes, per (row, kv head) unit u, 8 slots at stamps + 8u: 0 first CTA
 * entry (atomic min), 1 last CTA done with its tiles (atomic max), 2 last
 * split part arrived, 3 local merge done, 4 partial pushed to every peer
 * (split-KV across GPUs), 5 every peer's partial seen, 6 result stored.
 * The caller fills slot 0 with all ones (and 1.. with zeros) before the
 * launch.  Not for production launches: the stamps cost atomics.
 */
int nvqsa_set_stamp_buffer(void* stamps);

/*
 * Same computation as nvqsa_sparse_attention, for callers that cannot
 * allocate device memory: code that runs where cudaMalloc is unavailable or
 * forbidden (a host that hands this library only fixed, pre-registered
 * buffers, a real-time or embedded serving loop with a no-allocation rule, a
 * plugin whose framework owns every allocation).  It takes no workspace
 * argument and allocates nothing; the split-KV partials live in a static
 * device buffer of NVQSA_NOALLOC_SCRATCH_BYTES (16 MiB) that every device
 * loading this library keeps for the life of the process.
 *
 * Limit: problems whose split-KV partials need more than
 * NVQSA_NOALLOC_SCRATCH_BYTES (nvqsa_sparse_attention_workspace_size reports
 * the need; about splits * rows * query_heads * 1 KiB) are rejected with
 * NVQSA_ERR_SCRATCH_LIMIT before anything is launched.
 * The first call on each device looks up the buffer's device address; make
 * that first call outside any stream capture.  The looked-up address is kept
 * for the process: after a cudaDeviceReset of that device it is stale, so
 * do not call this entry point on a device that was reset.  All calls on a
 * device share
 * the one buffer, so calls that may overlap on the GPU (different streams
 * without ordering between them) race and must be serialised by the caller.
 * Nothing in the buffer needs to start at zero: each call zeroes its
 * arrival counters on its stream and writes every partial it later reads.
 * No counterpart in the reference.
 */
#define NVQSA_NOALLOC_SCRATCH_BYTES (16u << 20)

int nvqsa_sparse_attention_noalloc(
    const void* query, int64_t q_stride_row, int64_t q_stride_head,
    const void* key_data, int64_t kd_stride_block, int64_t kd_stride_token, int64_t kd_stride_head,
    const void* key_scale, int64_t ks_stride_block, int64_t ks_stride_token, int64_t ks_stride_head,
    const void* value_data, int64_t vd_stride_block, int64_t vd_stride_token, int64_t vd_stride_head,
    const void* value_scale, int64_t vs_stride_block, int64_t vs_stride_token, int64_t vs_stride_head,
    int64_t num_blocks, int64_t page_size, int32_t kv_heads,
    float key_global_scale, float value_global_scale,
    const int32_t* logical_indices, int64_t topk,
    const int32_t* block_table, int64_t num_requests, int64_t table_width,
    const int32_t* token_to_request,
    void* output, int64_t o_stride_row, int64_t o_stride_head,
    int64_t rows, int32_t query_heads, int32_t head_dim, void* stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* NVFP4_QSA_H_ */
