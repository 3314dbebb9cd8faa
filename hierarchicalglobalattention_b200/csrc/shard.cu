// Unpack of a multi-GPU prefill's all-gathered buffers into the whole-sequence row layout.
//
// After the all-gather, rank r's contribution starts at recv + r * rank_stride.  One part of it
// (chunk_k, group_k, K rows or V rows) sits at part_offset: `pieces` blocks of [bk][rows][row_bytes]
// (bk = batch * kv_heads), piece j of rank r holding the rows of sequence block dst_block[r][j].
// The destination is [bk][world * pieces blocks][rows][row_bytes].  One warp copies one row with
// 16-byte loads and stores (row_bytes is a multiple of 16).
#include "hga_common.cuh"

namespace hga {

constexpr int kMaxShardBlocks = 128;
struct BlockMap {
  int32_t dst[kMaxShardBlocks];
};

__global__ void __launch_bounds__(256) shard_unpack_kernel(const unsigned char* __restrict__ recv, int64_t rank_stride,
                                                           int64_t part_offset, int world, int pieces, BlockMap map,
                                                           int64_t bk, int64_t rows, int64_t row_bytes,
                                                           unsigned char* __restrict__ dst) {
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t total = (int64_t)world * pieces * bk * rows;
  if (warp >= total) return;
  const int64_t row = warp % rows;
  const int64_t t = warp / rows;
  const int64_t b = t % bk;
  const int64_t rj = t / bk;  // r * pieces + j
  const int r = (int)(rj / pieces), j = (int)(rj % pieces);
  const uint4* s = reinterpret_cast<const uint4*>(recv + r * rank_stride + part_offset +
                                                  (((int64_t)j * bk + b) * rows + row) * row_bytes);
  uint4* d = reinterpret_cast<uint4*>(dst + ((b * (int64_t)(world * pieces) + map.dst[rj]) * rows + row) * row_bytes);
  for (int64_t i = lane; i < row_bytes / 16; i += 32) d[i] = s[i];
}

cudaError_t launch_shard_unpack(const void* recv, int64_t rank_stride, int64_t part_offset, int world, int pieces,
                                const int32_t* dst_block, int64_t bk, int64_t rows, int64_t row_bytes, void* dst,
                                cudaStream_t st) {
  BlockMap map;
  for (int i = 0; i < world * pieces; ++i) map.dst[i] = dst_block[i];
  const int64_t warps = (int64_t)world * pieces * bk * rows;
  if (warps == 0) return cudaSuccess;
  const int64_t blocks = (warps * 32 + 255) / 256;
  shard_unpack_kernel<<<(unsigned)blocks, 256, 0, st>>>((const unsigned char*)recv, rank_stride, part_offset, world,
                                                        pieces, map, bk, rows, row_bytes, (unsigned char*)dst);
  return cudaGetLastError();
}

}  // namespace hga
