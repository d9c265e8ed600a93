// Host launchers of the tile-list builder kernels (tiles.cu).
#pragma once

#include <algorithm>
#include <cstdint>
#include <cuda_runtime.h>

namespace fwn {

// 32-bit words of the per-block key-block bitmap for a mask with n_cols columns.
int tiles_bitmap_words(int n_cols);

// tile_ptr[nqb + 1] (exclusive scan of per-block tile counts; `counts` is nqb ints of workspace).
cudaError_t launch_tiles_count(const int32_t* indptr, const int32_t* indices, int n_rows, int n_cols, int block_q,
                               int32_t* tile_ptr, int32_t* counts, cudaStream_t stream);

cudaError_t launch_tiles_fill(const int32_t* indptr, const int32_t* indices, int n_rows, int n_cols, int block_q,
                              const int32_t* tile_ptr, int32_t* tile_kb, uint32_t* tile_bits, cudaStream_t stream);

cudaError_t launch_pair_count(const int32_t* ptr, const int32_t* kb, int n_blocks, int n_cols, int32_t* ptr2,
                              int32_t* counts, cudaStream_t stream);

cudaError_t launch_pair_fill(const int32_t* ptr, const int32_t* kb, const uint32_t* bits, int n_blocks, int n_cols,
                             const int32_t* ptr2, int32_t* kb2, uint32_t* bits2, cudaStream_t stream);

// Gathered list from a 128-row list: pass 1 (ptr_g via per-block tile counts) and pass 2 (cols, bits).
// max_sub = the largest number of tiles of one block in the 128-row list.
cudaError_t launch_gather_count(const int32_t* ptr2, const uint32_t* bits2, int n_blocks, int32_t* ptr_g,
                                int32_t* counts, cudaStream_t stream);
cudaError_t launch_gather_fill(const int32_t* ptr2, const int32_t* kb2, const uint32_t* bits2, int n_blocks,
                               int max_sub, const int32_t* ptr_g, int32_t* cols_g, uint32_t* bits_g,
                               cudaStream_t stream);

// Hilbert-curve codes of (lat, lon) points in degrees (bits per axis <= 20); INT64_MAX for non-finite.
cudaError_t launch_hilbert_codes(const double* lat_deg, const double* lon_deg, int n, int bits, long long* codes,
                                 cudaStream_t stream);

// ptr[0] = 0, ptr[i + 1] = ptr[i] + counts[i] for i < n (one CTA).
cudaError_t launch_exclusive_scan(const int32_t* counts, int n, int32_t* ptr, cudaStream_t stream);

// k-hop reach (khop.cu): uint32 words per bitset row of n_cols columns (a multiple of 4).
int bitset_words(int n_cols);

// reach[n, bitset_words(n)] = nodes within `hops` edges of each node (self included), or with include_self
// false the end nodes of walks of exactly `hops` edges; scratch is the same size. indptr / indices: CSR of the
// graph (any column order, duplicates allowed).
cudaError_t launch_khop(const int32_t* indptr, const int32_t* indices, int n, int hops, uint32_t* reach,
                        uint32_t* scratch, cudaStream_t stream, bool include_self);

// CSR of a bitset matrix: indptr[n_rows + 1] (counts: n_rows ints of workspace), then ascending indices.
cudaError_t launch_bitset_csr_count(const uint32_t* bits, int n_rows, int n_cols, int32_t* indptr, int32_t* counts,
                                    cudaStream_t stream);
cudaError_t launch_bitset_csr_fill(const uint32_t* bits, int n_rows, int n_cols, const int32_t* indptr,
                                   int32_t* indices, cudaStream_t stream);

// Conditioned LayerNorm (norm.cu): out = LN(x) * (1 + scale[s]) + offset[s], s = row / rows_per_sample,
// scale_offset [samples, 2 d]; d in {128, 256, 512, 1024}; out bf16 or float32; out_node (nullable) maps each
// row within its sample to its output row; residual (nullable, bf16 [rows, d]) is first added into x in place.
cudaError_t launch_cond_layernorm(const float* x, float* x_out, int64_t rows, int d, int rows_per_sample,
                                  const int32_t* out_node, const float* so, float eps, void* out, bool bf16_out,
                                  const void* residual, cudaStream_t stream);
// Backward of the conditioned norm (x the normalised input): dx (+ dx_in), optional bf16 copy of dx, and the
// per-sample scale / offset gradients dso [samples, 2 d] through a workspace of per-CTA column partials.
size_t cond_layernorm_bwd_workspace(int64_t rows, int d, int rows_per_sample);
cudaError_t launch_cond_layernorm_bwd(const float* x, int64_t rows, int d, int rows_per_sample, const float* so,
                                      float eps, const void* dy, bool dy_bf16, const float* dx_in, float* dx,
                                      void* dx_bf16, float* dso, void* ws, cudaStream_t stream);

// Interaction-network pieces (gnn.cu): h = act(E + S[snd] + R[rcv] + bias) (bf16), and out[i] = norm * sum over the
// receiver's sorted edge run of LN(m[e]) (+ residual[i]).
cudaError_t launch_gather_add_act(const void* e_proj, const void* s_proj, const int32_t* snd, const void* r_proj,
                                  const int32_t* rcv, const void* bias, int64_t rows, int h, bool swish, void* out,
                                  cudaStream_t stream);
cudaError_t launch_ln_segment_sum(const void* m, const int32_t* seg, int64_t n_out, int f, const void* gamma,
                                  const void* beta, float eps, float norm, const float* residual, void* out,
                                  bool bf16_out, cudaStream_t stream);

}  // namespace fwn
