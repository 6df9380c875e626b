// Tile-packed weight layout used by every quantized matvec kernel.
//
// The reference stores a quantized matrix in its flat row-major form (Q1:
// LSB-first sign bits + one fp16 scale per group; Q4: 8 nibbles per u32 +
// scale + bias per group; nnmetal/src/metal.zig:235-469).  At load time this
// library re-orders the SAME bits into tiles so that
//   * one 16-byte load per lane gives a complete int8 MMA A-fragment after a
//     single AND per register (Q1: four 1-bit weights -> four u8 {0, 2^j};
//     Q4: two nibbles of two rows per byte),
//   * a row tile's data for one scale group, including its scales (and
//     biases), is one contiguous "segment" fetched by one bulk copy.
// No value is changed: unpack(pack(x)) == x bit for bit (tested).
//
// Geometry (all formats): row tile = 128 rows, K chunk = 32 columns,
// group size gs a multiple of 32 dividing K.  Lane L = 4*g + t (g = L>>2,
// t = L&3) owns 4 little-endian u32 words ("regs" r = 0..3) per chunk.
//
// Q1 (chunk block = 512 B):  bit (j + 8*i) of word r of lane (g,t) holds the
//   weight at row 16*j + g + 8*(r&1), column 4*t + i + 16*(r>>1) of the chunk.
//   Scales per (tile, group): 8 x 16 fp16, value v of lane-group g belongs to
//   row 16*(v>>1) + g + 8*(v&1).  Segment = (gs/32)*512 + 256 bytes.
// Q4 (chunk block = 4 subtiles x 512 B = 2048 B): in subtile u, byte i of word
//   r of lane (g,t) holds the low nibble of row 32u + g + 8*(r&1) and the high
//   nibble of row 32u + 16 + g + 8*(r&1), column 4*t + i + 16*(r>>1).
//   Scales/biases per (tile, group): 8 x (16 scales, 16 biases) u16, value
//   v = 4u + w of lane-group g belongs to row 32u + {g, g+8, 16+g, 24+g}[w].
//   Segment = (gs/32)*2048 + 512 bytes.
// Rows >= M are zero padded (scale 0, bias 0).
//
// A packed matrix may interleave SUB matrices of equal shape per group
// ([tile][group][sub][segment]) so that one CTA fetches e.g. the gate and up
// rows of the same tile with one copy.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __CUDACC__
#define NNZ_HD __host__ __device__
#else
#define NNZ_HD
#endif

namespace nnz {

enum Fmt : int { FMT_Q1 = 0, FMT_Q4 = 1 };

constexpr int kTileRows = 128;
constexpr int kChunk = 32;

NNZ_HD inline constexpr uint32_t chunk_bytes(int fmt) { return fmt == FMT_Q1 ? 512u : 2048u; }
NNZ_HD inline constexpr uint32_t scale_bytes(int fmt) { return fmt == FMT_Q1 ? 256u : 512u; }
NNZ_HD inline constexpr uint32_t seg_bytes(int fmt, uint32_t gs) {
  return (gs / kChunk) * chunk_bytes(fmt) + scale_bytes(fmt);
}
NNZ_HD inline constexpr uint32_t num_tiles(uint32_t M) { return (M + kTileRows - 1) / kTileRows; }
NNZ_HD inline constexpr size_t packed_bytes(int fmt, uint32_t M, uint32_t K, uint32_t gs, uint32_t sub) {
  return static_cast<size_t>(num_tiles(M)) * (K / gs) * sub * seg_bytes(fmt, gs);
}

// Host packing / unpacking (packing.cpp).  `weight` is the reference's flat
// buffer (Q1: M*K/8 bytes; Q4: M*K/8 u32 words), scales/biases u16 per group.
// `sub_index`/`sub` place this matrix as sub-matrix `sub_index` of `sub`.
int pack_host(int fmt, const void* weight, const uint16_t* scales, const uint16_t* biases,
              uint32_t M, uint32_t K, uint32_t gs, uint32_t sub, uint32_t sub_index, void* out,
              int nthreads);
int unpack_host(int fmt, const void* packed, uint32_t M, uint32_t K, uint32_t gs, uint32_t sub,
                uint32_t sub_index, void* weight, uint16_t* scales, uint16_t* biases);
// Tensor-parallel shard of a flat [M][K] matrix: rows [lo, hi) (axis 0) or
// columns [lo, hi) (axis 1, lo and hi multiples of gs) into flat outputs of
// the shard's own shape.  biases may be null (Q1).
int shard_host(int fmt, int axis, const void* weight, const uint16_t* scales, const uint16_t* biases,
               uint32_t M, uint32_t K, uint32_t gs, uint32_t lo, uint32_t hi, void* w_out,
               uint16_t* s_out, uint16_t* b_out);

}  // namespace nnz
