// Unpack of a multi-GPU prefill's all-gathered buffers into the whole-sequence row layout.
//
// After the all-gather, rank r's contribution starts at recv + r * rank_stride.  One part of it
// (chunk_k, group_k, K rows or V rows) sits at part_offset: `pieces` blocks of [bk][rows][row_bytes]
// (bk = batch * kv_heads), piece j of rank r holding the rows of sequence block dst_block[r][j].
// The destination is [bk][world * pieces blocks][rows][row_bytes].  Each source block is one
// contiguous run of rows in both buffers and is copied in 16-byte pieces (row_bytes is a multiple
// of 16).
#include "hga_common.cuh"

namespace hga {

constexpr int kMaxShardBlocks = 128;
struct BlockMap {
  int32_t dst[kMaxShardBlocks];
};

// grid.y = (r * pieces + j) * bk + b: one source block of rows; grid.x strides over its 16-byte
// pieces (rows * row_bytes / 16, contiguous in both source and destination): plain coalesced
// copies, 4 pieces in flight per thread, no per-row index arithmetic.
__global__ void __launch_bounds__(256) shard_unpack_kernel(const unsigned char* __restrict__ recv, int64_t rank_stride,
                                                           int64_t part_offset, int pieces, BlockMap map, int64_t bk,
                                                           int64_t rows, int64_t row_bytes, int world_pieces,
                                                           unsigned char* __restrict__ dst) {
  const int64_t y = blockIdx.y;
  const int64_t b = y % bk;
  const int rj = (int)(y / bk);  // r * pieces + j
  const int r = rj / pieces, j = rj % pieces;
  const uint4* s = reinterpret_cast<const uint4*>(recv + r * rank_stride + part_offset + (((int64_t)j * bk + b) * rows) * row_bytes);
  uint4* d = reinterpret_cast<uint4*>(dst + ((b * (int64_t)world_pieces + map.dst[rj]) * rows) * row_bytes);
  const int64_t n = rows * row_bytes / 16;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * step < n; i += 4 * step) {
    const uint4 a0 = s[i], a1 = s[i + step], a2 = s[i + 2 * step], a3 = s[i + 3 * step];
    d[i] = a0; d[i + step] = a1; d[i + 2 * step] = a2; d[i + 3 * step] = a3;
  }
  for (; i < n; i += step) d[i] = s[i];
}

cudaError_t launch_shard_unpack(const void* recv, int64_t rank_stride, int64_t part_offset, int world, int pieces,
                                const int32_t* dst_block, int64_t bk, int64_t rows, int64_t row_bytes, void* dst,
                                cudaStream_t st) {
  BlockMap map;
  for (int i = 0; i < world * pieces; ++i) map.dst[i] = dst_block[i];
  const int64_t nblk = (int64_t)world * pieces * bk;
  const int64_t n = rows * row_bytes / 16;
  if (nblk == 0 || n == 0) return cudaSuccess;
  if (nblk > 65535) return cudaErrorInvalidConfiguration;
  // about 8 CTAs of 256 threads per SM in total, each thread moving 4 pieces per round
  int64_t gx = (148 * 8 + nblk - 1) / nblk;
  const int64_t gx_max = (n + 256 * 4 - 1) / (256 * 4);
  gx = gx < 1 ? 1 : (gx > gx_max ? gx_max : gx);
  shard_unpack_kernel<<<dim3((unsigned)gx, (unsigned)nblk), 256, 0, st>>>((const unsigned char*)recv, rank_stride,
                                                                          part_offset, pieces, map, bk, rows, row_bytes,
                                                                          world * pieces, (unsigned char*)dst);
  return cudaGetLastError();
}

}  // namespace hga
