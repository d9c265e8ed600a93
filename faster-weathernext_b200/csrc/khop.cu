// Device-side neighbourhood masks: the k-hop reach of a graph as a bitset matrix, and its CSR.
//
// Replaces the host sparse matrix power `adj_mat ** attention_k_hop` (src/faster_weathernext/patch.py:209)
// whose nonzero pattern is the attention mask. reach_0 = I, reach_{s+1}[i] = reach_s[i] | OR_{j in adj(i)}
// reach_s[j]; after `hops` steps row i holds every node within `hops` edges of i, i.e. the pattern of
// (adj + I) ** hops. Rows are bitsets of `words` uint32 (bit c of word w = column 32 w + c), so one
// step reads (1 + degree) rows per row: HBM-bound, coalesced 16-byte loads, no atomics. The walk variant
// drops the `reach_s[i] |` term: after `length` steps row i holds the end nodes of the walks of exactly
// `length` edges from i, the nonzero pattern of adj ** length itself (what the reference's matrix power gives
// for any adjacency, with or without self edges).
//
// The CSR conversion writes ascending column indices per row (warp-wide popcount prefix over each run of
// 32 words), which is what the tile-list builder and scipy's sorted CSR hold.
#include "tiles.cuh"

namespace fwn {

namespace {

constexpr int kStepThreads = 128;

__global__ void __launch_bounds__(256) bitset_identity_kernel(uint32_t* __restrict__ bits, int n, int words) {
  const size_t total = static_cast<size_t>(n) * words;
  for (size_t e = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; e < total;
       e += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(e / words), w = static_cast<int>(e % words);
    bits[e] = (w == (i >> 5)) ? (1u << (i & 31)) : 0u;
  }
}

// One CTA per row: dst[i] = (kSelf ? src[i] : 0) | OR of src[j] over the row's neighbours (indices outside
// [0, n) ignored).
template <bool kSelf>
__global__ void __launch_bounds__(kStepThreads) khop_step_kernel(const int32_t* __restrict__ indptr,
                                                                const int32_t* __restrict__ indices, int n,
                                                                int words, const uint4* __restrict__ src,
                                                                uint4* __restrict__ dst) {
  __shared__ int nbr[kStepThreads];
  const int i = blockIdx.x;
  const int vw = words / 4;  // uint4 per row (words is a multiple of 4)
  const int e0 = indptr[i], e1 = indptr[i + 1];
  const uint4* own = src + static_cast<size_t>(i) * vw;
  // Both loops have the same trip count in every thread (the barriers below are reached by the whole CTA);
  // threads past the row's end only help stage neighbour ids.
  for (int v0 = 0; v0 < vw; v0 += kStepThreads) {
    const int v = v0 + threadIdx.x;
    const bool active = v < vw;
    uint4 acc = (kSelf && active) ? own[v] : make_uint4(0, 0, 0, 0);
    for (int base = e0; base < e1; base += kStepThreads) {
      // Neighbour ids are staged per batch of kStepThreads edges.
      __syncthreads();
      const int e = base + threadIdx.x;
      nbr[threadIdx.x] = e < e1 ? indices[e] : -1;
      __syncthreads();
      const int cnt = min(kStepThreads, e1 - base);
      if (active) {
        for (int k = 0; k < cnt; ++k) {
          const int j = nbr[k];
          if (j < 0 || j >= n) continue;
          const uint4 x = src[static_cast<size_t>(j) * vw + v];
          acc.x |= x.x;
          acc.y |= x.y;
          acc.z |= x.z;
          acc.w |= x.w;
        }
      }
    }
    if (active) dst[static_cast<size_t>(i) * vw + v] = acc;
  }
}

// counts[r] = popcount of row r's columns < n_cols (one warp per row).
__global__ void __launch_bounds__(256) bitset_count_kernel(const uint32_t* __restrict__ bits, int n_rows, int n_cols,
                                                           int words, int32_t* __restrict__ counts) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (r >= n_rows) return;
  const uint32_t* row = bits + static_cast<size_t>(r) * words;
  const int used = (n_cols + 31) / 32;
  int c = 0;
  for (int w = lane; w < used; w += 32) {
    uint32_t x = row[w];
    if (w == used - 1 && (n_cols & 31)) x &= (1u << (n_cols & 31)) - 1u;
    c += __popc(x);
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) c += __shfl_xor_sync(0xffffffffu, c, d);
  if (lane == 0) counts[r] = c;
}

// indices[indptr[r] ...] = the set columns of row r, ascending (one warp per row).
__global__ void __launch_bounds__(256) bitset_fill_kernel(const uint32_t* __restrict__ bits, int n_rows, int n_cols,
                                                          int words, const int32_t* __restrict__ indptr,
                                                          int32_t* __restrict__ indices) {
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (r >= n_rows) return;
  const uint32_t* row = bits + static_cast<size_t>(r) * words;
  const int used = (n_cols + 31) / 32;
  int out = indptr[r];
  for (int base = 0; base < used; base += 32) {
    const int w = base + lane;
    uint32_t x = w < used ? row[w] : 0u;
    if (w == used - 1 && (n_cols & 31)) x &= (1u << (n_cols & 31)) - 1u;
    const int c = __popc(x);
    int incl = c;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    int pos = out + incl - c;
    while (x) {
      const int b = __ffs(x) - 1;
      indices[pos++] = 32 * w + b;
      x &= x - 1u;
    }
    out += __shfl_sync(0xffffffffu, incl, 31);
  }
}

}  // namespace

int bitset_words(int n_cols) { return ((n_cols + 31) / 32 + 3) / 4 * 4; }

cudaError_t launch_khop(const int32_t* indptr, const int32_t* indices, int n, int hops, uint32_t* reach,
                        uint32_t* scratch, cudaStream_t stream, bool include_self) {
  if (n <= 0) return cudaSuccess;
  const int words = bitset_words(n);
  // Ping-pong so that the last step writes `reach`.
  uint32_t* a = (hops % 2 == 0) ? reach : scratch;
  uint32_t* b = (hops % 2 == 0) ? scratch : reach;
  const size_t total = static_cast<size_t>(n) * words;
  const int grid = static_cast<int>(std::min<size_t>((total + 255) / 256, 148 * 32));
  bitset_identity_kernel<<<grid, 256, 0, stream>>>(a, n, words);
  for (int s = 0; s < hops; ++s) {
    if (include_self)
      khop_step_kernel<true><<<n, kStepThreads, 0, stream>>>(indptr, indices, n, words,
                                                             reinterpret_cast<const uint4*>(a), reinterpret_cast<uint4*>(b));
    else
      khop_step_kernel<false><<<n, kStepThreads, 0, stream>>>(indptr, indices, n, words,
                                                              reinterpret_cast<const uint4*>(a), reinterpret_cast<uint4*>(b));
    std::swap(a, b);
  }
  return cudaGetLastError();
}

cudaError_t launch_bitset_csr_count(const uint32_t* bits, int n_rows, int n_cols, int32_t* indptr, int32_t* counts,
                                    cudaStream_t stream) {
  const int words = bitset_words(n_cols);
  if (n_rows > 0) bitset_count_kernel<<<(n_rows * 32 + 255) / 256, 256, 0, stream>>>(bits, n_rows, n_cols, words, counts);
  launch_exclusive_scan(counts, n_rows, indptr, stream);
  return cudaGetLastError();
}

cudaError_t launch_bitset_csr_fill(const uint32_t* bits, int n_rows, int n_cols, const int32_t* indptr,
                                   int32_t* indices, cudaStream_t stream) {
  const int words = bitset_words(n_cols);
  if (n_rows > 0)
    bitset_fill_kernel<<<(n_rows * 32 + 255) / 256, 256, 0, stream>>>(bits, n_rows, n_cols, words, indptr, indices);
  return cudaGetLastError();
}

}  // namespace fwn
