// Host-side repacking of GGUF Q8_0 blocks into the packed device format.
//
// GGUF stores a row-major [n, k] Q8_0 tensor as n*k/32 records of 34 bytes
// (`<f2 scale><32 x i8>`, parakeet_cuda/gguf.py:63-65,135-149). The packed
// format regroups them per tile of 128 (layout-permuted) rows and per 32-wide
// K block into 4352-byte records:
//   bytes [   0, 2048): int8 values k in [0, 16) of rows 0..127, 16 bytes per row
//   bytes [2048, 4096): int8 values k in [16, 32) of rows 0..127
//   bytes [4096, 4352): the 128 fp16 scales
// so that a warp reading 16 bytes per lane touches 512 contiguous bytes and a
// whole record is one 16-byte-aligned bulk copy. Values and scales are moved
// bit for bit; nothing is re-quantised.
#include <cstring>

#include "pq8.h"

namespace {

struct Header {
  uint32_t magic, version;
  int32_t n, k, layout, n_tiles, k_blocks, out_cols;
};
constexpr uint32_t kMagic = 0x50385150u;

bool layout_ok(int n, int layout) {
  switch (layout) {
    case PQ8_LAYOUT_ROWS: return n >= 1;
    case PQ8_LAYOUT_GLU: return n >= 2 && n % 2 == 0;
    case PQ8_LAYOUT_GATES4: return n >= 4 && n % 4 == 0;
    default: return false;
  }
}

int out_cols(int n, int layout) {
  return layout == PQ8_LAYOUT_GLU ? n / 2 : layout == PQ8_LAYOUT_GATES4 ? n / 4 : n;
}

// Source row for packed row p; -1 for padding. Mirrors map_row() in pq8_device.cuh.
int source_row(int layout, int n, int p) {
  const int t = p >> 7, r = p & 127;
  if (layout == PQ8_LAYOUT_ROWS) return p < n ? p : -1;
  if (layout == PQ8_LAYOUT_GLU) {
    const int h = n / 2, w = r >> 5, l = r & 31, j = t * 64 + w * 16 + (l & 15);
    if (j >= h) return -1;
    return l < 16 ? j : h + j;
  }
  const int h = n / 4, g = r >> 5, u = t * 32 + (r & 31);
  return u < h ? g * h + u : -1;
}

}  // namespace

extern "C" int pq8_packed_size(int n, int k, int layout, size_t* bytes) {
  if (bytes == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (k <= 0 || k % 32 != 0 || !layout_ok(n, layout)) return PQ8_ERR_UNSUPPORTED_SHAPE;
  const size_t n_tiles = (static_cast<size_t>(n) + PQ8_TILE_ROWS - 1) / PQ8_TILE_ROWS;
  *bytes = PQ8_HEADER_BYTES + n_tiles * static_cast<size_t>(k / 32) * PQ8_RECORD_BYTES;
  return PQ8_OK;
}

extern "C" int pq8_pack_q8_0_part(const void* gguf_blocks, int n, int k_src, int k_total, int k_offset,
                                  int layout, void* packed) {
  if (gguf_blocks == nullptr || packed == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (k_src <= 0 || k_src % 32 || k_total <= 0 || k_total % 32 || k_offset < 0 || k_offset % 32 ||
      k_offset + k_src > k_total || !layout_ok(n, layout))
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  size_t total = 0;
  pq8_packed_size(n, k_total, layout, &total);
  auto* out = static_cast<unsigned char*>(packed);
  Header* h = reinterpret_cast<Header*>(out);
  const int n_tiles = (n + PQ8_TILE_ROWS - 1) / PQ8_TILE_ROWS;
  const int kb_total = k_total / 32, kb_src = k_src / 32, kb_off = k_offset / 32;
  if (k_offset == 0) {
    std::memset(out, 0, total);
    h->magic = kMagic;
    h->version = 1;
    h->n = n;
    h->k = k_total;
    h->layout = layout;
    h->n_tiles = n_tiles;
    h->k_blocks = kb_total;
    h->out_cols = out_cols(n, layout);
  } else if (h->magic != kMagic || h->n != n || h->k != k_total || h->layout != layout) {
    return PQ8_ERR_LAYOUT;
  }
  const auto* src = static_cast<const unsigned char*>(gguf_blocks);
  unsigned char* data = out + PQ8_HEADER_BYTES;
  for (int t = 0; t < n_tiles; ++t) {
    for (int r = 0; r < PQ8_TILE_ROWS; ++r) {
      const int s = source_row(layout, n, t * PQ8_TILE_ROWS + r);
      if (s < 0) continue;
      const unsigned char* row = src + static_cast<size_t>(s) * kb_src * 34;
      for (int kb = 0; kb < kb_src; ++kb) {
        const unsigned char* blk = row + static_cast<size_t>(kb) * 34;
        unsigned char* rec = data + (static_cast<size_t>(t) * kb_total + kb_off + kb) * PQ8_RECORD_BYTES;
        std::memcpy(rec + r * 16, blk + 2, 16);
        std::memcpy(rec + 2048 + r * 16, blk + 18, 16);
        std::memcpy(rec + 4096 + r * 2, blk, 2);
      }
    }
  }
  return PQ8_OK;
}

extern "C" int pq8_pack_q8_0(const void* gguf_blocks, int n, int k, int layout, void* packed) {
  return pq8_pack_q8_0_part(gguf_blocks, n, k, k, 0, layout, packed);
}
