// layout.cuh -- device-resident data layouts shared by the host runtime and
// the kernels.
//
// Weights (written once by mxmoe_upload_experts):
//   W1 codes  [E][2*fp][Kp1/2]  E2M1 nibble pairs, rows regrouped into 64-row
//             blocks that alternate GLU / linear (row of GLU unit j at
//             w1_packed_row(j, 0), its linear partner at w1_packed_row(j, 1)),
//             so one 128-row tensor-core tile holds 64 complete GLU pairs.
//             fp = f rounded up to 64, Kp1 = d rounded up to 128 (zero codes).
//   W2 codes  [E][d][Kp2/2], Kp2 = fp rounded up to 128.
//   scales    E8M0 with the file offset removed, stored as 512-byte atoms that
//             the MMA's scale-factor TMEM layout reads directly:
//             atom (row block of 128, k chunk of 4 x 32 columns);
//             byte (r % 32) * 16 + (r / 32 % 4) * 4 + (kb % 4).  The two
//             atoms of one 256-row tile and k chunk are adjacent
//             (w_sf_offset), so a pipeline stage fetches them in one copy.
// Activations (per forward, rows = routed (token, expert) pairs sorted by
// expert, every expert segment padded to a multiple of 128 rows):
//   codes     [2 terms][rows][Kp] E4M3 (value = hi + lo, two block-scaled terms);
//             stacked tiles keep both terms of a tile in consecutive rows
//             instead (stacked_code_row)
//   scales    [terms][rows/R][Kp/128] atoms, same byte order as weights, with
//             R = min(N, 128) rows per atom for tile width N.
// FP4 decode tiles (kind::mxf4): the activation is a sum of four block-scaled
// E2M1 terms, packed two codes per byte like the weights, and the four terms
// of a 32-pair tile fill one 128-row operand (stacked4_code_row).
#pragma once
#include <cstdint>

namespace mxmoe {

constexpr int kTileK = 128;        // K elements per pipeline stage / TMA box
constexpr int kRowBlock = 128;     // rows per scale-factor atom
constexpr int kSfAtomBytes = 512;  // 128 rows x 4 scale bytes
constexpr int kGluBlock = 64;      // GLU/linear interleave granularity (rows)
constexpr int kTerms = 2;          // E4M3 terms per activation (hi, lo)

__host__ __device__ inline uint32_t round_up(uint32_t v, uint32_t m) { return (v + m - 1) / m * m; }

__host__ __device__ inline uint32_t sf_atom_byte(uint32_t row_in_block, uint32_t kb_in_chunk) {
  return (row_in_block & 31u) * 16u + ((row_in_block >> 5) & 3u) * 4u + (kb_in_chunk & 3u);
}

// Packed W1 row of GLU unit j (half = 0) or its linear partner (half = 1).
__host__ __device__ inline uint32_t w1_packed_row(uint32_t j, uint32_t half) {
  return (j / kGluBlock) * (2 * kGluBlock) + half * kGluBlock + (j % kGluBlock);
}

// Byte offset of the scale of (row, k block) inside an atom array laid out
// [row_blocks][k_chunks][512], one atom per `block_rows` rows (128 for
// weights; min(N, 128) for activations so that every N-row tile starts on an
// atom and its scale factors land in TMEM lanes 0..N-1).
__host__ __device__ inline uint64_t sf_offset(uint32_t row, uint32_t kb, uint32_t k_chunks,
                                              uint32_t block_rows = kRowBlock) {
  return (static_cast<uint64_t>(row / block_rows) * k_chunks + kb / 4) * kSfAtomBytes +
         sf_atom_byte(row % block_rows, kb % 4);
}

// Stacked activation tiles of PT pairs (PT = 16, 32 or 64), both terms in one
// 128-row MMA operand: pair j of the tile, term t, is operand row
// (j / 16) * 32 + 16 * t + j % 16, so every 32-lane TMEM sub-partition
// carries 16 pairs' hi rows followed by their lo rows (rows from 2 * PT on
// feed discarded accumulator rows).  Scales: one atom per tile and k chunk,
// operand row r at sf_atom_byte(r, kb).
__host__ __device__ inline uint32_t stacked_operand_row(uint32_t j, uint32_t term) {
  return (j / 16u) * 32u + 16u * term + j % 16u;
}
__host__ __device__ inline uint64_t stacked_sf_offset(uint32_t row, uint32_t term, uint32_t kb, uint32_t k_chunks,
                                                      uint32_t pt) {
  return (static_cast<uint64_t>(row / pt) * k_chunks + kb / 4) * kSfAtomBytes +
         sf_atom_byte(stacked_operand_row(row % pt, term), kb % 4);
}

// Weight scales: byte offset of (row, k block) in [row_pairs][k_chunks][2][512]
// (row pair = 256 rows; the rows' 128-row block picks the atom of the pair).
constexpr int kWSfPairBytes = 2 * kSfAtomBytes;
__host__ __device__ inline uint32_t w_sf_row_pairs(uint32_t rows) { return (rows + 255u) / 256u; }
__host__ __device__ inline uint64_t w_sf_offset(uint32_t row, uint32_t kb, uint32_t k_chunks) {
  return (static_cast<uint64_t>(row / 256u) * k_chunks + kb / 4) * kWSfPairBytes + ((row / 128u) & 1u) * kSfAtomBytes +
         sf_atom_byte(row % 128u, kb % 4);
}

// Stacked activation codes: pair pos, term t -> code row in one buffer of
// 2 x rows rows: a PT-pair tile occupies 2 * PT consecutive rows in operand
// order, so one TMA box of 2 * PT rows loads it.
__host__ __device__ inline uint32_t stacked_code_row(uint32_t pos, uint32_t term, uint32_t pt) {
  return (pos / pt) * (2u * pt) + stacked_operand_row(pos % pt, term);
}

// FP4 stacked tiles of PT <= 32 pairs, four E2M1 terms in one 128-row MMA
// operand: pair j, term t is operand row (j / 8) * 32 + 8 * t + j % 8, so
// every 32-lane TMEM sub-partition carries 8 pairs with their four terms in
// lanes L, L + 8, L + 16, L + 24.
constexpr int kF4Terms = 4;
constexpr int kF4PairTile = 32;       // widest FP4 tile (4 x 32 = 128 operand rows)
constexpr int kF4PairTileSmall = 16;  // 64 operand rows: half the activation bytes per stage
__host__ __device__ inline uint32_t stacked4_operand_row(uint32_t j, uint32_t term) {
  return (j / 8u) * 32u + 8u * term + j % 8u;
}
// Code row of (pair pos, term t) in a buffer of 4 x rows rows of Kp/2 bytes:
// a tile's 4 * PT rows are consecutive, in operand order.
__host__ __device__ inline uint32_t stacked4_code_row(uint32_t pos, uint32_t term, uint32_t pt) {
  return (pos / pt) * (4u * pt) + stacked4_operand_row(pos % pt, term);
}
// Scale byte of (pair pos, term t, k block kb): one atom per tile and 128-K
// chunk, [tiles][k_chunks][512], so a stage's two chunks are adjacent.
__host__ __device__ inline uint64_t stacked4_sf_offset(uint32_t pos, uint32_t term, uint32_t kb, uint32_t k_chunks,
                                                       uint32_t pt) {
  return (static_cast<uint64_t>(pos / pt) * k_chunks + kb / 4) * kSfAtomBytes +
         sf_atom_byte(stacked4_operand_row(pos % pt, term), kb % 4);
}

}  // namespace mxmoe
