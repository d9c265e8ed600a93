/*
 * fwn_attn.h — C ABI of libfwn_attn.so, the B200 (sm_100a) block-sparse masked flash attention of
 * faster-weathernext's mesh-transformer processor.
 *
 * Reference interfaces replaced (Raymondlol/Faster-WeatherNext v0.2.0):
 *   fwn_tiles_count / fwn_tiles_fill      <- pallas_attn.build_tile_mask   (src/faster_weathernext/pallas_attn.py:85-109)
 *   fwn_tiles_pair_count / _fill          <- (no counterpart: derives the 128-query-row list the kernels walk
 *                                             from build_tile_mask's 64-row list; see pallas_attn.py:112-141)
 *   fwn_attn_fwd                          <- pallas_attn._forward / _kernel (pallas_attn.py:112-141, 235-257)
 *                                             and the custom-VJP forward rule _attention_fwd (pallas_attn.py:267-271)
 *   fwn_attn_bwd                          <- pallas_attn._attention_bwd with _bwd_dq_kernel / _bwd_dkv_kernel
 *                                             (pallas_attn.py:161-215, 274-311)
 *   fwn_attn_desc                         <- the static arguments of tiled_flash_attention (pallas_attn.py:317-354):
 *                                             shapes, `scale`, precision preset (TF32 / 3xTF32) and layout
 *
 * Conventions
 *   - Every pointer is device memory owned by the caller; nothing here allocates, frees or synchronises
 *     (except fwn_device_error, which synchronises the stream to read the device error word).
 *   - Calls are stateless and may be issued concurrently on different streams.
 *   - Tensors q, k, v, o, d_o, dq, dk, dv use the reference's public layout [batch, n, heads, head_dim] with
 *     head_dim contiguous and arbitrary element strides for batch / node / head (multiples of 16 bytes):
 *     one set for the inputs q, k, v, one for o, d_o, dq, dk, dv.
 *   - lse is float32 [batch, heads, fwn_lse_rows(n)] (natural-log log-sum-exp of the scaled logits).
 *   - Tile lists follow build_tile_mask: block b owns tiles ptr[b]..ptr[b+1]-1 in ascending key-block
 *     order; tile t covers keys kb[t]*32 + [0, 32); bit j of bits[t*rows + r] allows (row b*rows + r,
 *     key kb[t]*32 + j). The attention kernels take the 128-row ("paired") form.
 *   - Errors are returned as fwn_status; fwn_last_error_string() describes the last failure of the calling
 *     thread.
 */
#ifndef FWN_ATTN_H_
#define FWN_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FWN_API __attribute__((visibility("default")))
#else
#define FWN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum fwn_status {
  FWN_OK = 0,
  FWN_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad shape, stride or alignment */
  FWN_ERR_UNSUPPORTED = 2,      /* head_dim / dtype / mode combination not built */
  FWN_ERR_WORKSPACE = 3,        /* workspace missing or too small */
  FWN_ERR_LAUNCH = 4,           /* CUDA runtime / driver error */
  FWN_ERR_DEVICE_TIMEOUT = 5,   /* a bounded device-side wait expired; the kernel returned early */
  FWN_ERR_NO_DEVICE = 6         /* no sm_100 device is current */
} fwn_status;

typedef enum fwn_dtype { FWN_DTYPE_BF16 = 0, FWN_DTYPE_F32 = 1 } fwn_dtype;

/* Arithmetic of the attention MMAs. BF16 takes bf16 tensors; TF32 and TF32X3 take float32 tensors.
 * TF32 <-> the reference's default precision (DotAlgorithmPreset.TF32_TF32_F32, pallas_attn.py:342);
 * TF32X3 <-> jax.default_matmul_precision("highest") (TF32_TF32_F32_X3, pallas_attn.py:338-340). */
typedef enum fwn_mode { FWN_MODE_BF16 = 0, FWN_MODE_TF32 = 1, FWN_MODE_TF32X3 = 2 } fwn_mode;

typedef struct fwn_attn_desc {
  int32_t batch;
  int32_t heads;
  int32_t n;          /* nodes (rows of q and k) */
  int32_t head_dim;   /* 64 or 128 */
  float scale;        /* softmax scale; the reference passes key_size ** -0.5 (patch.py:174) */
  int32_t dtype;      /* fwn_dtype of q, k, v, o, d_o, dq, dk, dv */
  int32_t mode;       /* fwn_mode */
  int32_t flags;      /* fwn_desc_flags bits; 0: the fields up to out_stride_h are all that is read */
  int64_t stride_b;   /* element strides of q, k, v ([batch, n, heads, head_dim], head_dim contiguous) */
  int64_t stride_n;
  int64_t stride_h;
  int64_t out_stride_b; /* element strides of o, d_o, and of dq, dk, dv unless FWN_DESC_GRAD_STRIDES is set */
  int64_t out_stride_n;
  int64_t out_stride_h;
  int64_t grad_stride_b; /* with FWN_DESC_GRAD_STRIDES only: element strides of dq, dk, dv, e.g. views of one */
  int64_t grad_stride_n; /* [batch, n, heads, 3, head_dim] gradient of a fused q / k / v projection's output */
  int64_t grad_stride_h; /* (the reference's patch.py:165-177 projections), written in place by the backward */
} fwn_attn_desc;

/* fwn_attn_desc.flags. A caller built against a header without the grad_stride fields passes flags = 0 and its
 * shorter struct is read only up to out_stride_h. */
typedef enum fwn_desc_flags { FWN_DESC_GRAD_STRIDES = 1 } fwn_desc_flags;

typedef struct fwn_tile_list {
  const int32_t* ptr;   /* [n_blocks + 1] */
  const int32_t* kb;    /* [n_tiles] */
  const uint32_t* bits; /* [n_tiles * block_rows] */
  int32_t n_blocks;
  int32_t n_tiles;
  int32_t block_rows;   /* 64: build_tile_mask layout; 128: paired or gathered layout (attention kernels) */
  int32_t n_cols;       /* columns of the mask (keys); key blocks are < ceil(n_cols / 32) */
  const int32_t* cols;  /* NULL, or [n_tiles * 32]: gathered list, slot j of tile t is column cols[t*32 + j]
                           (kb unused). Gathered lists need q/k/v (and o/d_o) laid out so that (batch, node,
                           head) rows form one strided 2D view: node-major (stride_n = heads * stride_h,
                           stride_b = n * stride_n) or head-major (stride_h = n * stride_n, stride_b =
                           heads * stride_h). */
} fwn_tile_list;

/* Version string of the library build. */
FWN_API const char* fwn_version(void);

/* Description of the last error returned to the calling thread ("" if none). */
FWN_API const char* fwn_last_error_string(void);

/* Synchronises `stream`, reads and clears the device error word written by bounded waits (and by
 * fwn_gemm_bf16_gather on an index out of range). *code receives 0, FWN_ERR_DEVICE_TIMEOUT, or FWN_ERR_INVALID_ARGUMENT
 * for such an index. */
FWN_API fwn_status fwn_device_error(void* stream, int32_t* code);

/* Rows of the lse buffer per (batch, head): n rounded up to a multiple of 128. */
FWN_API int32_t fwn_lse_rows(int32_t n);

/* ---- tile-list builder (replaces pallas_attn.build_tile_mask, pallas_attn.py:85-109) -------------------- */

/* Workspace bytes fwn_tiles_count needs for an [n_rows, n_cols] mask with block_q-row blocks. */
FWN_API fwn_status fwn_tiles_workspace_size(int32_t n_rows, int32_t n_cols, int32_t block_q, size_t* bytes);

/* Pass 1: tile_ptr[ceil(n_rows/block_q) + 1] from the CSR (indptr[n_rows+1], indices[nnz]) of a boolean
 * mask (duplicates allowed, any column order). The tile count is tile_ptr[last]. block_q in {64, 128};
 * key tiles are 32 columns (one uint32 word per row per tile). */
FWN_API fwn_status fwn_tiles_count(const int32_t* indptr, const int32_t* indices, int32_t n_rows, int32_t n_cols,
                           int32_t block_q, int32_t* tile_ptr, void* ws, size_t ws_bytes, void* stream);

/* Pass 2: tile_kb[n_tiles] and tile_bits[n_tiles * block_q] for the tile_ptr of pass 1. Bit-exact with
 * build_tile_mask for block_q = 64. The transposed list (pallas_attn.py:351-352, patch.py:215-218) is
 * the same two passes over the CSR of the transposed mask. */
FWN_API fwn_status fwn_tiles_fill(const int32_t* indptr, const int32_t* indices, int32_t n_rows, int32_t n_cols,
                          int32_t block_q, const int32_t* tile_ptr, int32_t* tile_kb, uint32_t* tile_bits,
                          void* stream);

/* Paired 128-row list from a 64-row list: block p = rows of blocks 2p and 2p+1; its tiles are the union
 * of their key blocks (ascending); words of rows 0-63 come from block 2p, rows 64-127 from 2p+1 (0 where
 * that block lacks the key block). pass 1 writes ptr2[ceil(n_blocks/2) + 1]; pass 2 kb2 and bits2. */
FWN_API fwn_status fwn_tiles_pair_count(const fwn_tile_list* tiles64, int32_t* ptr2, void* ws, size_t ws_bytes,
                                void* stream);
FWN_API fwn_status fwn_tiles_pair_fill(const fwn_tile_list* tiles64, const int32_t* ptr2, int32_t* kb2,
                               uint32_t* bits2, void* stream);

/* Gathered list from a 128-row list (no counterpart in the reference; derived from build_tile_mask's list):
 * per block, the distinct columns its rows may attend to, ascending, packed into tiles of 32 slots (the
 * last tile padded with the block's last column, whose padding slots carry no bits). Pass 1 writes
 * ptr_g[n_blocks + 1]; pass 2 cols_g[T_g * 32] and bits_g[T_g * 128]. max_block_tiles >= the largest
 * ptr[b+1] - ptr[b] of the 128-row list (at most 40,960). */
FWN_API fwn_status fwn_tiles_gather_count(const fwn_tile_list* tiles128, int32_t* ptr_g, void* ws, size_t ws_bytes,
                                          void* stream);
FWN_API fwn_status fwn_tiles_gather_fill(const fwn_tile_list* tiles128, int32_t max_block_tiles,
                                         const int32_t* ptr_g, int32_t* cols_g, uint32_t* bits_g, void* stream);

/* Hilbert-curve codes (3D, `bits` per axis, 1..20) of unit-sphere points given in degrees; non-finite
 * points get INT64_MAX. A stable argsort of the codes is pallas_attn.hilbert_order (pallas_attn.py:41-82). */
FWN_API fwn_status fwn_hilbert_codes(const double* lat_deg, const double* lon_deg, int32_t n, int32_t bits,
                                     int64_t* codes, void* stream);

/* ---- neighbourhood masks on the device ------------------------------------------------------------- */

/* uint32 words per row of a bitset matrix with n_cols columns (bit c of word w = column 32 w + c); a
 * multiple of 4, so every row starts on a 16-byte boundary. */
FWN_API int32_t fwn_bitset_words(int32_t n_cols);

/* k-hop neighbourhood: reach[n * fwn_bitset_words(n)] row i = every node within `hops` edges of node i,
 * self included, i.e. the nonzero pattern of (adj + I) ** hops. Replaces the host sparse matrix power
 * `adj_mat ** attention_k_hop` (src/faster_weathernext/patch.py:209); for a mesh adjacency (which has
 * triangles) and hops >= 2 the two patterns are equal. indptr[n + 1] / indices: CSR of adj (any column
 * order, duplicates allowed). scratch has reach's size. 0 <= hops <= 4096. */
FWN_API fwn_status fwn_khop_bitset(const int32_t* indptr, const int32_t* indices, int32_t n, int32_t hops,
                                   uint32_t* reach, uint32_t* scratch, void* stream);

/* Matrix-power pattern: reach row i = the end nodes of the walks of exactly `length` edges of adj from node i,
 * the nonzero pattern of adj ** length for any adjacency (self edges count only where adj has them; length 0
 * gives the identity). This is `adj_mat ** attention_k_hop` of the reference's _transformer_init
 * (src/faster_weathernext/patch.py:209) exactly; for an adjacency with every self edge it equals
 * fwn_khop_bitset. Same arguments and limits as fwn_khop_bitset. */
FWN_API fwn_status fwn_walk_bitset(const int32_t* indptr, const int32_t* indices, int32_t n, int32_t length,
                                   uint32_t* reach, uint32_t* scratch, void* stream);

/* CSR of a bitset matrix [n_rows, fwn_bitset_words(n_cols)] (columns >= n_cols ignored), in two passes as
 * the tile builder: pass 1 writes indptr[n_rows + 1] (ws: n_rows int32; nnz = indptr[n_rows]); pass 2
 * writes indices[nnz], ascending per row. n_rows * n_cols must be below 2^31. The result feeds
 * fwn_tiles_count / fwn_tiles_fill directly. */
FWN_API fwn_status fwn_bitset_csr_count(const uint32_t* bits, int32_t n_rows, int32_t n_cols, int32_t* indptr,
                                        void* ws, size_t ws_bytes, void* stream);
FWN_API fwn_status fwn_bitset_csr_fill(const uint32_t* bits, int32_t n_rows, int32_t n_cols, const int32_t* indptr,
                                       int32_t* indices, void* stream);

/* ---- the processor around the attention ---------------------------------------------------------------- */

/* Conditioned LayerNorm of the pre-LN blocks (src/faster_weathernext/patch.py:238-252, 288-290: LayerNorm without
 * scale / offset, then the norm conditioning's per-sample scale and offset):
 *   out[r, :] = (x[r, :] - mean) / sqrt(var + eps) * (1 + scale_offset[s, :d]) + scale_offset[s, d:],
 *   s = r / rows_per_sample. x float32 [rows, d] contiguous, d in {128, 256, 512, 1024}; scale_offset float32
 *   [rows / rows_per_sample, 2 d]; out [rows, d] in `out_dtype` (FWN_DTYPE_BF16 or FWN_DTYPE_F32). */
FWN_API fwn_status fwn_cond_layernorm(const float* x, int64_t rows, int32_t d, int32_t rows_per_sample,
                                      const float* scale_offset, float eps, void* out, int32_t out_dtype,
                                      void* stream);

/* The same norm with the node un-permutation of the reference's transformer fused into the store
 * (src/faster_weathernext/patch.py:291-292, x = take(x, argsort(perm)) after the final norm): row i of each sample
 * goes to row out_node[i] of that sample, out_node int32 [rows_per_sample], a permutation of
 * [0, rows_per_sample) (pass the forward permutation perm itself). An entry outside that range drops its row. */
FWN_API fwn_status fwn_cond_layernorm_scatter(const float* x, int64_t rows, int32_t d, int32_t rows_per_sample,
                                              const int32_t* out_node, const float* scale_offset, float eps,
                                              void* out, int32_t out_dtype, void* stream);

/* The pre-LN block's residual add fused into the next norm (src/faster_weathernext/patch.py:238-252, `x = x + f(h)`
 * followed by the next LayerNorm): x[r, :] += residual[r, :] in place (x float32 [rows, d], residual bf16 [rows, d],
 * the sub-block's output), then out = the conditioned LayerNorm of the sum, as fwn_cond_layernorm (or, with out_node
 * non-null, fwn_cond_layernorm_scatter). One pass over the rows instead of an add and a norm. */
FWN_API fwn_status fwn_cond_layernorm_residual(float* x, const void* residual, int64_t rows, int32_t d,
                                               int32_t rows_per_sample, const int32_t* out_node,
                                               const float* scale_offset, float eps, void* out, int32_t out_dtype,
                                               void* stream);

/* Out-of-place form for the training path (autograd keeps the block's input): x_out = x + residual (x float32, residual
 * bf16, x_out float32, all [rows, d]; x_out may be x), out = the conditioned LayerNorm of x_out as fwn_cond_layernorm. */
FWN_API fwn_status fwn_cond_layernorm_add(const float* x, const void* residual, float* x_out, int64_t rows, int32_t d,
                                          int32_t rows_per_sample, const float* scale_offset, float eps, void* out,
                                          int32_t out_dtype, void* stream);

/* Backward of the conditioned LayerNorm (the VJP the reference's training path takes through the blocks' norms under
 * jax.grad, src/faster_weathernext/patch.py:238-252, 288-290), x the norm's input (after any residual add), dy the
 * gradient of out ([rows, d] in dy_dtype, bf16 or float32):
 *   g = dy (1 + scale[s]),  xhat = (x - mean) rstd,
 *   dx[r, :] = rstd (g - mean(g) - xhat mean(g xhat)) + dx_in[r, :]     (dx_in float32 or NULL; dx may be dx_in)
 *   dscale_offset[s, :d] = sum over the sample's rows of dy xhat,  dscale_offset[s, d:] = sum of dy   (float32)
 * dx_bf16 (bf16 [rows, d] or NULL) receives a bf16 copy of dx: the gradient of a bf16 residual that was added into x.
 * d in {128, 256, 512}. The per-sample sums are taken in a fixed order (per-CTA partials in `workspace`, then one
 * reduction kernel): deterministic. workspace: fwn_cond_layernorm_bwd_workspace bytes, 16-byte aligned. */
FWN_API size_t fwn_cond_layernorm_bwd_workspace(int64_t rows, int32_t d, int32_t rows_per_sample);
FWN_API fwn_status fwn_cond_layernorm_bwd(const float* x, int64_t rows, int32_t d, int32_t rows_per_sample,
                                          const float* scale_offset, float eps, const void* dy, int32_t dy_dtype,
                                          const float* dx_in, float* dx, void* dx_bf16, float* dscale_offset,
                                          void* workspace, size_t workspace_bytes, void* stream);

/* Projections around the attention (src/faster_weathernext/patch.py:165-177, 250-252: q / k / v, mha_final, the
 * MLP): c[m, n] = act(a[m, k] b[k, n] + bias[n]), a row-major bf16 [m, k], b given transposed as bt row-major bf16
 * [n, k] (the weight with k contiguous), bias bf16 [n] or NULL, c row-major bf16 [m, n]; float32 accumulation on the
 * tensor cores. n a multiple of 256, k a multiple of 64, pointers 16-byte aligned. act: FWN_ACT_NONE or
 * FWN_ACT_GELU_TANH (0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3))), jax.nn.gelu's default form). */
typedef enum fwn_act {
  FWN_ACT_NONE = 0,
  FWN_ACT_GELU_TANH = 1,
  FWN_ACT_SWISH = 2,
  FWN_ACT_GELU_TANH_AUX = 3,  /* fwn_gemm_bf16_aux: c = GELU(x) and aux = x (x = a b + bias), both bf16 [m, n] */
  FWN_ACT_GELU_TANH_GRAD = 4  /* fwn_gemm_bf16_aux: c = x GELU'(aux), aux the bf16 [m, n] input GELU was applied to */
} fwn_act;
FWN_API fwn_status fwn_gemm_bf16(const void* a, const void* bt, const void* bias, void* c, int64_t m, int32_t n,
                                 int32_t k, int32_t act, void* stream);

/* The MLP of the processor's training path (src/faster_weathernext/patch.py:250-252 under jax.grad): the same GEMM
 * with an aux tensor (bf16 [m, n], 16-byte aligned). act FWN_ACT_GELU_TANH_AUX: c = GELU(x), aux = x, x = a b + bias
 * (the forward, keeping the pre-activation for the backward); FWN_ACT_GELU_TANH_GRAD: c = x GELU'(aux), x = a b (+ bias)
 * (the backward: a = the gradient of the MLP's output, bt = the down-projection weight as stored, [hidden, d], so x is
 * the gradient of the activation, and c the gradient of the pre-activation). FWN_ACT_NONE / FWN_ACT_GELU_TANH ignore
 * aux. */
FWN_API fwn_status fwn_gemm_bf16_aux(const void* a, const void* bt, const void* bias, void* c, void* aux, int64_t m,
                                     int32_t n, int32_t k, int32_t act, void* stream);

/* The interaction network's MLP input layers (src/faster_weathernext/patch.py:347-509: the edge MLP over (edge, sender,
 * receiver) features with the pre-gather projections, pre_gather_{senders,receivers,edges}_for_edges_fn; the node MLP
 * over (node, aggregate)): the same GEMM with rows of two more tensors added before the activation,
 *   c[i, :] = act(a[i, :] bt^T + bias + add0[idx0[i], :] + add1[idx1[i], :]),
 * add0 / add1 bf16 [rows0 / rows1, n] row-major (either may be NULL), idx0 / idx1 int32 [m] (NULL: row i itself, which
 * then needs rows >= m); act FWN_ACT_NONE or FWN_ACT_SWISH (x sigmoid(x)). One pass instead of the GEMM's output
 * written and read back by a separate gather-add. An index outside [0, rows) adds nothing to its row and is reported by
 * fwn_device_error as FWN_ERR_INVALID_ARGUMENT. */
FWN_API fwn_status fwn_gemm_bf16_gather(const void* a, const void* bt, const void* bias, void* c, const void* add0,
                                        const int32_t* idx0, int64_t rows0, const void* add1, const int32_t* idx1,
                                        int64_t rows1, int64_t m, int32_t n, int32_t k, int32_t act, void* stream);

/* ---- grid <-> mesh interaction networks -------------------------------------------------------------------
 * The blocked GNNs of the encoder / decoder (src/faster_weathernext/patch.py:347-509, ChunkedDeepGNN: edge MLP on
 * (edge, sender, receiver) features with the first layer's matmul applied per node before the gather, a sorted
 * segment-sum of the messages into the receivers, a node MLP); the matmuls run on fwn_gemm_bf16.
 *
 * h[e, :] = act(e_proj[e, :] + s_proj[senders[e], :] + r_proj[receivers[e], :] + bias), bf16 [rows, h] each (h a
 * multiple of 8); any of e_proj / s_proj / r_proj / bias may be NULL (left out), senders / receivers may be NULL
 * (row e itself). act: FWN_ACT_NONE or FWN_ACT_SWISH (x sigmoid(x)). */
FWN_API fwn_status fwn_gnn_gather_add_act(const void* e_proj, const void* s_proj, const int32_t* senders,
                                          const void* r_proj, const int32_t* receivers, const void* bias, int64_t rows,
                                          int32_t h, int32_t act, void* out, void* stream);

/* out[i, :] = norm * sum_{e = seg_ptr[i]}^{seg_ptr[i+1]-1} LN(m[e, :]) (+ residual[i, :]): LayerNorm of each message
 * row (eps, scale gamma, offset beta: bf16 [f]) summed over the receiver's edges, which the caller sorts by receiver
 * (seg_ptr [n_out + 1], the CSR offsets of the runs; NULL: row i alone, for a node MLP's output norm); residual
 * float32 [n_out, f] or NULL; out [n_out, f] float32 or bf16 (out_dtype). m bf16 [edges, f], f in {256, 512, 1024}.
 * One warp per receiver, no atomics: deterministic. */
FWN_API fwn_status fwn_gnn_ln_segment_sum(const void* m, const int32_t* seg_ptr, int64_t n_out, int32_t f,
                                          const void* gamma, const void* beta, float eps, float norm,
                                          const float* residual, void* out, int32_t out_dtype, void* stream);

/* ---- attention --------------------------------------------------------------------------------------- */

/* Forward: o = softmax(mask(q k^T * scale)) v over the tiles of `tiles` (128-row list); lse (nullable)
 * receives m + log(l) per row, the residual of the custom-VJP forward rule. Rows with no allowed key get
 * o = 0 and lse = -inf. */
FWN_API fwn_status fwn_attn_fwd(const fwn_attn_desc* desc, const void* q, const void* k, const void* v,
                        const fwn_tile_list* tiles, void* o, float* lse, void* stream);

/* Workspace bytes of fwn_attn_bwd (the per-row delta = rowsum(o * d_o), float32). */
FWN_API fwn_status fwn_attn_bwd_workspace_size(const fwn_attn_desc* desc, size_t* bytes);

/* Backward: dq over `tiles` (the forward's 128-row list), dk/dv over `tiles_t` (the 128-row list of the
 * transposed mask; pass `tiles` again for a symmetric mask, pallas_attn.py:351-352). */
FWN_API fwn_status fwn_attn_bwd(const fwn_attn_desc* desc, const void* q, const void* k, const void* v,
                        const void* o, const float* lse, const void* d_o, const fwn_tile_list* tiles,
                        const fwn_tile_list* tiles_t, void* dq, void* dk, void* dv, void* ws,
                        size_t ws_bytes, void* stream);

/* The three launches of fwn_attn_bwd, one by one (same arguments; ws holds delta between them):
 *   fwn_attn_bwd_delta  delta = rowsum(o * d_o)                      <- pallas_attn.py:278 (XLA reduction)
 *   fwn_attn_bwd_dq     dq over `tiles`                              <- _bwd_dq_kernel, pallas_attn.py:161-184, 286-295
 *   fwn_attn_bwd_dkv    dk, dv over `tiles_t`                        <- _bwd_dkv_kernel, pallas_attn.py:187-215, 297-311 */
FWN_API fwn_status fwn_attn_bwd_delta(const fwn_attn_desc* desc, const void* o, const void* d_o, void* ws,
                                      size_t ws_bytes, void* stream);
FWN_API fwn_status fwn_attn_bwd_dq(const fwn_attn_desc* desc, const void* q, const void* k, const void* v,
                                   const float* lse, const void* d_o, const fwn_tile_list* tiles, void* dq,
                                   const void* ws, size_t ws_bytes, void* stream);
FWN_API fwn_status fwn_attn_bwd_dkv(const fwn_attn_desc* desc, const void* q, const void* k, const void* v,
                                    const float* lse, const void* d_o, const fwn_tile_list* tiles_t, void* dk,
                                    void* dv, const void* ws, size_t ws_bytes, void* stream);

/* ---- backward without a caller workspace ---------------------------------------------------------------
 * No counterpart in the reference. fwn_attn_bwd needs a workspace for the per-row delta = rowsum(o * d_o);
 * this variant keeps delta in a fixed device array inside the library instead, for callers that cannot
 * allocate device memory at the point of the call: an XLA / jax.ffi custom-call handler whose buffers are
 * all owned by XLA, code that runs while another component holds the allocator, or a loop that must not
 * take cudaMalloc's implicit device synchronisation. The caller still passes every input and output.
 *   - Capacity: batch * heads * fwn_lse_rows(n) <= FWN_NOALLOC_DELTA_ROWS (4 MiB of float32); larger
 *     problems are rejected with FWN_ERR_WORKSPACE.
 *   - The first call on each device looks up the array's device address (with that device current);
 *     make that first call before any stream capture. The address is kept for the life of the process: after
 *     cudaDeviceReset on a device (which unloads the library's device code; a later call may find it loaded
 *     at another address) this entry point must not be called again on that device.
 *   - The array is shared by every call on a device and keeps the last call's contents; each call
 *     rewrites all of the rows it reads. Calls that overlap on the GPU (different streams, no ordering)
 *     race on it: order them, or use fwn_attn_bwd with separate workspaces.
 *   - Nothing is allocated, freed or synchronised. */
#define FWN_NOALLOC_DELTA_ROWS (1 << 20)
FWN_API fwn_status fwn_attn_bwd_noalloc(const fwn_attn_desc* desc, const void* q, const void* k, const void* v,
                                        const void* o, const float* lse, const void* d_o,
                                        const fwn_tile_list* tiles, const fwn_tile_list* tiles_t, void* dq,
                                        void* dk, void* dv, void* stream);

/* ---- failure detection test -----------------------------------------------------------------------------
 * No counterpart in the reference. fwn_attn_fwd with one input copy left out on purpose, so that a bounded
 * device-side wait expires: the producer of CTA 0 does not issue the first K / V load of its first work item,
 * the MMA warp's wait on it gives up after wait_limit_ns (1e5 .. 2e9 ns; every other wait of the launch has
 * the same bound), the CTA's other roles leave at their next wait, the producer waits for the copies it did
 * issue, the CTA frees its tensor memory and returns, and the device error word reads
 * FWN_ERR_DEVICE_TIMEOUT (fwn_device_error). No copy, MMA or tensor-memory allocation is left behind, so the
 * context stays usable; o / lse are incomplete. Only the narrow bf16 head_dim-64 forward (sparse lists). */
FWN_API fwn_status fwn_test_attn_fwd_timeout(const fwn_attn_desc* desc, const void* q, const void* k, const void* v,
                                             const fwn_tile_list* tiles, void* o, float* lse, uint64_t wait_limit_ns,
                                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FWN_ATTN_H_ */
