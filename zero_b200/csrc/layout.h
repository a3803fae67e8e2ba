// layout.h — device layout of a registered Q4_0 / Q8_0 matmul tensor.
//
// Rows are taken four at a time (the 4-row groups of the .smodel-v2 X4
// format, tools/silicatepack.py:982-1022); each group is one contiguous
// "group stream" on the device so that fused projections can concatenate or
// interleave whole groups.  A group stream is a sequence of chunks of up to
// kChunkBlocks consecutive 32-element blocks.  A chunk of nb blocks holds:
//
//   P planes of nb 16-byte entries, then one scale plane of nb 8-byte entries
//   (the four rows' fp16 block scales d0..d3), padded to a multiple of 16 B.
//
//   Q4_0: P = 4, plane r entry j = the 16 nibble bytes (qs) of row r, block j
//         (byte i: low nibble = element i, high nibble = element i + 16).
//   Q8_0: P = 8, plane 2r + h entry j = int8 elements 16h .. 16h+15 of row r,
//         block j.
//
// Every chunk, and so every group stream, is a multiple of 16 bytes, so each
// chunk is one legal 1-D bulk copy.  A warp that gives lane j block j reads
// every plane with one conflict-free 16-byte shared-memory load per lane.
// The byte count per block equals the X4 format's (72 B / 136 B per 4 rows);
// only an odd-length last chunk carries 8 bytes of padding.
#pragma once

#include <stdint.h>

#include "../../include/zgpu.h"

#ifdef __CUDACC__
#define ZGPU_HD __host__ __device__ __forceinline__
#else
#define ZGPU_HD inline
#endif

namespace zgpu {

constexpr uint32_t kChunkBlocks = 32;

ZGPU_HD uint32_t plane_count(uint32_t quant) { return quant == ZGPU_Q4_0 ? 4u : 8u; }

// Bytes of a chunk holding nb blocks.
ZGPU_HD uint64_t chunk_bytes(uint32_t quant, uint32_t nb) {
  return static_cast<uint64_t>(plane_count(quant)) * nb * 16u + ((nb * 8u + 15u) & ~15u);
}

// Blocks in chunk c of a row of bpr blocks.
ZGPU_HD uint32_t chunk_blocks(uint64_t bpr, uint64_t c) {
  const uint64_t rest = bpr - c * kChunkBlocks;
  return rest < kChunkBlocks ? static_cast<uint32_t>(rest) : kChunkBlocks;
}

// Byte offset of chunk c inside a group stream (all chunks before the last
// are full).
ZGPU_HD uint64_t chunk_offset(uint32_t quant, uint64_t c) { return c * chunk_bytes(quant, kChunkBlocks); }

// Bytes of one group stream for rows of bpr blocks (a multiple of 16).
ZGPU_HD uint64_t group_stream_bytes(uint32_t quant, uint64_t bpr) {
  const uint64_t full = bpr / kChunkBlocks, rem = bpr % kChunkBlocks;
  return full * chunk_bytes(quant, kChunkBlocks) + (rem ? chunk_bytes(quant, static_cast<uint32_t>(rem)) : 0);
}

// Offset of block b's entry in plane p, and of its scale entry, inside a
// group stream.
ZGPU_HD uint64_t plane_entry(uint32_t quant, uint64_t bpr, uint64_t b, uint32_t p) {
  const uint64_t c = b / kChunkBlocks, j = b % kChunkBlocks;
  return chunk_offset(quant, c) + static_cast<uint64_t>(p) * chunk_blocks(bpr, c) * 16u + j * 16u;
}
ZGPU_HD uint64_t scale_entry(uint32_t quant, uint64_t bpr, uint64_t b) {
  const uint64_t c = b / kChunkBlocks, j = b % kChunkBlocks;
  return chunk_offset(quant, c) + static_cast<uint64_t>(plane_count(quant)) * chunk_blocks(bpr, c) * 16u + j * 8u;
}

}  // namespace zgpu
