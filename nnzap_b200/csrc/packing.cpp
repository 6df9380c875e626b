// Host-side conversion between the reference's flat quantized layout and
// the tile-packed layout described in packing.h.  Pure integer work; runs at
// model load on all host cores.
#include "packing.h"

#include <string.h>

#include <algorithm>
#include <thread>
#include <vector>

namespace nnz {
namespace {

// spread4[n]: bit i of n -> bit 8*i (i = 0..3).
struct Spread4 {
  uint32_t v[16];
  Spread4() {
    for (uint32_t n = 0; n < 16; ++n) {
      uint32_t w = 0;
      for (uint32_t i = 0; i < 4; ++i) w |= ((n >> i) & 1u) << (8 * i);
      v[n] = w;
    }
  }
};
const Spread4 kSpread;

inline uint32_t q1_nib(const uint8_t* bits, uint64_t flat) {  // flat % 4 == 0
  return (bits[flat >> 3] >> (flat & 7)) & 0xFu;
}
inline uint32_t q4_quad(const uint32_t* words, uint64_t flat) {  // 4 nibbles, flat % 4 == 0
  return (words[flat >> 3] >> (4 * (flat & 7))) & 0xFFFFu;
}

void pack_tiles(int fmt, const void* weight, const uint16_t* scales, const uint16_t* biases,
                uint32_t M, uint32_t K, uint32_t gs, uint32_t sub, uint32_t si, uint8_t* out,
                uint32_t t0, uint32_t t1) {
  const uint32_t groups = K / gs, cpg = gs / kChunk, seg = seg_bytes(fmt, gs);
  const uint32_t spr = K / gs;  // scales per row
  for (uint32_t T = t0; T < t1; ++T) {
    for (uint32_t G = 0; G < groups; ++G) {
      uint8_t* base = out + (static_cast<size_t>(T * groups + G) * sub + si) * seg;
      for (uint32_t cc = 0; cc < cpg; ++cc) {
        const uint32_t kc = G * cpg + cc;
        for (uint32_t L = 0; L < 32; ++L) {
          const uint32_t g = L >> 2, t = L & 3;
          for (uint32_t r = 0; r < 4; ++r) {
            const uint32_t col0 = kc * kChunk + 4 * t + 16 * (r >> 1);
            if (fmt == FMT_Q1) {
              const uint8_t* bits = static_cast<const uint8_t*>(weight);
              uint32_t w = 0;
              for (uint32_t j = 0; j < 8; ++j) {
                const uint32_t row = T * kTileRows + 16 * j + g + 8 * (r & 1);
                if (row < M) w |= kSpread.v[q1_nib(bits, static_cast<uint64_t>(row) * K + col0)] << j;
              }
              memcpy(base + cc * 512 + L * 16 + r * 4, &w, 4);
            } else {
              const uint32_t* words = static_cast<const uint32_t*>(weight);
              for (uint32_t u = 0; u < 4; ++u) {
                const uint32_t ra = T * kTileRows + 32 * u + g + 8 * (r & 1), rb = ra + 16;
                const uint32_t qa = ra < M ? q4_quad(words, static_cast<uint64_t>(ra) * K + col0) : 0;
                const uint32_t qb = rb < M ? q4_quad(words, static_cast<uint64_t>(rb) * K + col0) : 0;
                uint32_t w = 0;
                for (uint32_t i = 0; i < 4; ++i)
                  w |= (((qa >> (4 * i)) & 0xFu) | (((qb >> (4 * i)) & 0xFu) << 4)) << (8 * i);
                memcpy(base + cc * 2048 + u * 512 + L * 16 + r * 4, &w, 4);
              }
            }
          }
        }
      }
      uint16_t* sc = reinterpret_cast<uint16_t*>(base + cpg * chunk_bytes(fmt));
      for (uint32_t g = 0; g < 8; ++g) {
        for (uint32_t v = 0; v < 16; ++v) {
          if (fmt == FMT_Q1) {
            const uint32_t row = T * kTileRows + 16 * (v >> 1) + g + 8 * (v & 1);
            sc[g * 16 + v] = row < M ? scales[static_cast<size_t>(row) * spr + G] : 0;
          } else {
            static const uint32_t off[4] = {0, 8, 16, 24};
            const uint32_t row = T * kTileRows + 32 * (v >> 2) + g + off[v & 3];
            sc[g * 32 + v] = row < M ? scales[static_cast<size_t>(row) * spr + G] : 0;
            sc[g * 32 + 16 + v] = row < M ? biases[static_cast<size_t>(row) * spr + G] : 0;
          }
        }
      }
    }
  }
}

}  // namespace

int pack_host(int fmt, const void* weight, const uint16_t* scales, const uint16_t* biases,
              uint32_t M, uint32_t K, uint32_t gs, uint32_t sub, uint32_t sub_index, void* out,
              int nthreads) {
  if ((fmt != FMT_Q1 && fmt != FMT_Q4) || !weight || !scales || !out) return -1;
  if (fmt == FMT_Q4 && !biases) return -1;
  if (M == 0 || K == 0 || gs == 0 || gs % kChunk || K % gs || sub == 0 || sub_index >= sub) return -1;
  const uint32_t tiles = num_tiles(M);
  if (nthreads <= 0) nthreads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  nthreads = static_cast<int>(std::min<uint32_t>(static_cast<uint32_t>(nthreads), tiles));
  uint8_t* o = static_cast<uint8_t*>(out);
  if (nthreads <= 1) {
    pack_tiles(fmt, weight, scales, biases, M, K, gs, sub, sub_index, o, 0, tiles);
    return 0;
  }
  std::vector<std::thread> th;
  for (int i = 0; i < nthreads; ++i) {
    const uint32_t a = static_cast<uint32_t>(static_cast<uint64_t>(tiles) * i / nthreads);
    const uint32_t b = static_cast<uint32_t>(static_cast<uint64_t>(tiles) * (i + 1) / nthreads);
    th.emplace_back(pack_tiles, fmt, weight, scales, biases, M, K, gs, sub, sub_index, o, a, b);
  }
  for (auto& t : th) t.join();
  return 0;
}

int unpack_host(int fmt, const void* packed, uint32_t M, uint32_t K, uint32_t gs, uint32_t sub,
                uint32_t si, void* weight, uint16_t* scales, uint16_t* biases) {
  if ((fmt != FMT_Q1 && fmt != FMT_Q4) || !packed || !weight || !scales) return -1;
  if (fmt == FMT_Q4 && !biases) return -1;
  if (M == 0 || K == 0 || gs == 0 || gs % kChunk || K % gs || sub == 0 || si >= sub) return -1;
  const uint8_t* in = static_cast<const uint8_t*>(packed);
  const uint32_t groups = K / gs, cpg = gs / kChunk, seg = seg_bytes(fmt, gs), spr = K / gs;
  if (fmt == FMT_Q1) memset(weight, 0, static_cast<size_t>(M) * K / 8);
  else memset(weight, 0, static_cast<size_t>(M) * K / 2);
  for (uint32_t T = 0; T < num_tiles(M); ++T) {
    for (uint32_t G = 0; G < groups; ++G) {
      const uint8_t* base = in + (static_cast<size_t>(T * groups + G) * sub + si) * seg;
      for (uint32_t cc = 0; cc < cpg; ++cc) {
        const uint32_t kc = G * cpg + cc;
        for (uint32_t L = 0; L < 32; ++L) {
          const uint32_t g = L >> 2, t = L & 3;
          for (uint32_t r = 0; r < 4; ++r) {
            const uint32_t col0 = kc * kChunk + 4 * t + 16 * (r >> 1);
            if (fmt == FMT_Q1) {
              uint32_t w;
              memcpy(&w, base + cc * 512 + L * 16 + r * 4, 4);
              uint8_t* bits = static_cast<uint8_t*>(weight);
              for (uint32_t j = 0; j < 8; ++j) {
                const uint32_t row = T * kTileRows + 16 * j + g + 8 * (r & 1);
                if (row >= M) continue;
                for (uint32_t i = 0; i < 4; ++i) {
                  const uint64_t f = static_cast<uint64_t>(row) * K + col0 + i;
                  if ((w >> (j + 8 * i)) & 1u) bits[f >> 3] |= static_cast<uint8_t>(1u << (f & 7));
                }
              }
            } else {
              uint32_t* words = static_cast<uint32_t*>(weight);
              for (uint32_t u = 0; u < 4; ++u) {
                uint32_t w;
                memcpy(&w, base + cc * 2048 + u * 512 + L * 16 + r * 4, 4);
                const uint32_t ra = T * kTileRows + 32 * u + g + 8 * (r & 1), rb = ra + 16;
                for (uint32_t i = 0; i < 4; ++i) {
                  const uint32_t byte = (w >> (8 * i)) & 0xFFu;
                  if (ra < M) {
                    const uint64_t f = static_cast<uint64_t>(ra) * K + col0 + i;
                    words[f >> 3] |= (byte & 0xFu) << (4 * (f & 7));
                  }
                  if (rb < M) {
                    const uint64_t f = static_cast<uint64_t>(rb) * K + col0 + i;
                    words[f >> 3] |= (byte >> 4) << (4 * (f & 7));
                  }
                }
              }
            }
          }
        }
      }
      const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + cpg * chunk_bytes(fmt));
      for (uint32_t g = 0; g < 8; ++g) {
        for (uint32_t v = 0; v < 16; ++v) {
          if (fmt == FMT_Q1) {
            const uint32_t row = T * kTileRows + 16 * (v >> 1) + g + 8 * (v & 1);
            if (row < M) scales[static_cast<size_t>(row) * spr + G] = sc[g * 16 + v];
          } else {
            static const uint32_t off[4] = {0, 8, 16, 24};
            const uint32_t row = T * kTileRows + 32 * (v >> 2) + g + off[v & 3];
            if (row < M) {
              scales[static_cast<size_t>(row) * spr + G] = sc[g * 32 + v];
              biases[static_cast<size_t>(row) * spr + G] = sc[g * 32 + 16 + v];
            }
          }
        }
      }
    }
  }
  return 0;
}

int shard_host(int fmt, int axis, const void* weight, const uint16_t* scales, const uint16_t* biases,
               uint32_t M, uint32_t K, uint32_t gs, uint32_t lo, uint32_t hi, void* w_out,
               uint16_t* s_out, uint16_t* b_out) {
  if ((fmt != FMT_Q1 && fmt != FMT_Q4) || gs == 0 || K % gs || lo >= hi || !weight || !scales || !w_out ||
      !s_out || (fmt == FMT_Q4 && (!biases || !b_out)))
    return -1;
  const uint8_t* w = static_cast<const uint8_t*>(weight);
  uint8_t* wo = static_cast<uint8_t*>(w_out);
  const size_t row_bytes = fmt == FMT_Q1 ? K / 8 : K / 2;   // 1 or 4 bits per weight
  const uint32_t ng = K / gs;
  if (axis == 0) {
    if (hi > M) return -1;
    const size_t n = hi - lo;
    memcpy(wo, w + lo * row_bytes, n * row_bytes);
    memcpy(s_out, scales + (size_t)lo * ng, n * ng * 2);
    if (fmt == FMT_Q4) memcpy(b_out, biases + (size_t)lo * ng, n * ng * 2);
    return 0;
  }
  if (axis != 1 || hi > K || lo % gs || hi % gs) return -1;
  const uint32_t kc = hi - lo, g0 = lo / gs, gn = kc / gs;
  const size_t b0 = fmt == FMT_Q1 ? lo / 8 : lo / 2, bn = fmt == FMT_Q1 ? kc / 8 : kc / 2;
  for (uint32_t r = 0; r < M; ++r) {
    memcpy(wo + (size_t)r * bn, w + (size_t)r * row_bytes + b0, bn);
    memcpy(s_out + (size_t)r * gn, scales + (size_t)r * ng + g0, (size_t)gn * 2);
    if (fmt == FMT_Q4) memcpy(b_out + (size_t)r * gn, biases + (size_t)r * ng + g0, (size_t)gn * 2);
  }
  return 0;
}

}  // namespace nnz
