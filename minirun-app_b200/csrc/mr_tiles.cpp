// mr_tiles.cpp — MNRNTIL1 tile containers: layout rules, header encoding and
// decoding, whole-tile reads with SHA-256 checks (host code only).
//
// Format and validation rules: Sources/StorageCore/Container/
// QuantizedTileContainer.swift — TileGeometry (:245-334), layout rules
// (:441-580), header fields (:739-784), decoding (:811-1001), digest check
// (:1153-1181). A reader re-derives every derivable field from the geometry
// and rejects any header that disagrees, so a corrupted or hand-edited header
// never steers a read.
#include "mr_tiles.h"

#include <errno.h>
#include <fcntl.h>
#include <stdio.h>
#include <string.h>
#include <sys/stat.h>
#include <unistd.h>

namespace mr {
namespace {

constexpr uint32_t kFlagBiases = MR_TILE_FLAG_BIASES;
constexpr uint32_t kFlagDigests = MR_TILE_FLAG_DIGESTS;
constexpr uint32_t kFlag2D = MR_TILE_FLAG_BLOCK_SCALES_2D;
constexpr uint32_t kFlagPadded = MR_TILE_FLAG_PADDED;
constexpr uint32_t kKnownFlags = kFlagBiases | kFlagDigests | kFlag2D | kFlagPadded;
constexpr int kV1Fields = 80, kV2Fields = 128, kV3Fields = 160;
constexpr int kDigestBytes = 32;

int digest_table_offset(int version) { return version >= 3 ? kV3Fields : kV2Fields; }

int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

int scale_elem_bytes(int dt) {
  switch (dt) {
    case MR_TILE_SCALE_E8M0: return 1;
    case MR_TILE_SCALE_F16:
    case MR_TILE_SCALE_BF16: return 2;
    case MR_TILE_SCALE_F32: return 4;
    default: return 0;
  }
}

const char* mode_name(int m) {
  switch (m) {
    case MR_TILE_MODE_MXFP4: return "mxfp4";
    case MR_TILE_MODE_AFFINE: return "affine";
    case MR_TILE_MODE_FP8_BLOCK: return "fp8-e4m3-block";
    default: return "unknown";
  }
}

bool has_biases(int mode) { return mode == MR_TILE_MODE_AFFINE; }
bool block_scales(int mode) { return mode == MR_TILE_MODE_FP8_BLOCK; }

std::string str(int64_t v) { return std::to_string(v); }

// little-endian field access
template <class T>
T get_le(const unsigned char* p) {
  T v = 0;
  for (size_t i = 0; i < sizeof(T); ++i) v |= (T)p[i] << (8 * i);
  return v;
}
template <class T>
void put_le(unsigned char* p, T v) {
  for (size_t i = 0; i < sizeof(T); ++i) p[i] = (unsigned char)((uint64_t)v >> (8 * i));
}

// ---------------------------------------------------------------- SHA-256
// FIPS 180-4, section 6.2: 64 rounds over 512-bit blocks; the round constants
// are the first 32 bits of the fractional parts of the cube roots of the first
// 64 primes, the initial hash the same for the square roots of the first 8.
constexpr uint32_t kSha[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4,
    0xab1c5ed5, 0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe,
    0x9bdc06a7, 0xc19bf174, 0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f,
    0x4a7484aa, 0x5cb0a9dc, 0x76f988da, 0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7,
    0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967, 0x27b70a85, 0x2e1b2138, 0x4d2c6dfc,
    0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85, 0xa2bfe8a1, 0xa81a664b,
    0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070, 0x19a4c116,
    0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7,
    0xc67178f2};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void sha_block(uint32_t h[8], const unsigned char* blk) {
  uint32_t w[64];
  for (int i = 0; i < 16; ++i)
    w[i] = (uint32_t)blk[4 * i] << 24 | (uint32_t)blk[4 * i + 1] << 16 |
           (uint32_t)blk[4 * i + 2] << 8 | (uint32_t)blk[4 * i + 3];
  for (int i = 16; i < 64; ++i) {
    const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
    const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
    w[i] = w[i - 16] + s0 + w[i - 7] + s1;
  }
  uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
  for (int i = 0; i < 64; ++i) {
    const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
    const uint32_t ch = (e & f) ^ (~e & g);
    const uint32_t t1 = k + S1 + ch + kSha[i] + w[i];
    const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
    const uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
    const uint32_t t2 = S0 + mj;
    k = g;
    g = f;
    f = e;
    e = d + t1;
    d = c;
    c = b;
    b = a;
    a = t1 + t2;
  }
  h[0] += a; h[1] += b; h[2] += c; h[3] += d;
  h[4] += e; h[5] += f; h[6] += g; h[7] += k;
}

}  // namespace

void sha256(const void* data, size_t n, unsigned char out[32]) {
  uint32_t h[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                   0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
  const unsigned char* p = static_cast<const unsigned char*>(data);
  size_t left = n;
  while (left >= 64) {
    sha_block(h, p);
    p += 64;
    left -= 64;
  }
  // padding: 0x80, zeros, then the message length in bits (big-endian)
  unsigned char tail[128] = {0};
  memcpy(tail, p, left);
  tail[left] = 0x80;
  const size_t tlen = left + 9 <= 64 ? 64 : 128;
  const uint64_t bits = (uint64_t)n * 8;
  for (int i = 0; i < 8; ++i) tail[tlen - 1 - i] = (unsigned char)(bits >> (8 * i));
  sha_block(h, tail);
  if (tlen == 128) sha_block(h, tail + 64);
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (unsigned char)(h[i] >> 24);
    out[4 * i + 1] = (unsigned char)(h[i] >> 16);
    out[4 * i + 2] = (unsigned char)(h[i] >> 8);
    out[4 * i + 3] = (unsigned char)h[i];
  }
}

bool tile_layout(mr_tile_layout* L, int64_t tile_count, bool has_digests, std::string& why) {
  const int mode = L->quant_mode;
  if (mode < MR_TILE_MODE_MXFP4 || mode > MR_TILE_MODE_FP8_BLOCK) {
    why = "unknown quantization mode " + str(mode);
    return false;
  }
  if (L->rows <= 0 || L->cols <= 0) {
    why = "rows and cols must be positive";
    return false;
  }
  if (tile_count <= 0) {
    why = "tileCount must be positive";
    return false;
  }
  if (L->bits != 4 && L->bits != 8) {
    why = "bits " + str(L->bits) + " is not supported; this format packs 4 or 8";
    return false;
  }
  if (L->group_size <= 0 || (L->group_size & (L->group_size - 1)) != 0) {
    why = "group size " + str(L->group_size) + " must be a positive power of two";
    return false;
  }
  if (mode == MR_TILE_MODE_MXFP4 && L->group_size != 32) {
    why = std::string(mode_name(mode)) + " fixes the group size at 32";
    return false;
  }
  const int esz = scale_elem_bytes(L->scale_dtype);
  if (esz == 0) {
    why = "unknown scale element type " + str(L->scale_dtype);
    return false;
  }
  if ((mode == MR_TILE_MODE_MXFP4 || mode == MR_TILE_MODE_FP8_BLOCK) &&
      L->scale_dtype != MR_TILE_SCALE_E8M0) {
    why = std::string(mode_name(mode)) + " scales are uint8-e8m0";
    return false;
  }
  if ((mode == MR_TILE_MODE_MXFP4 && L->bits != 4) ||
      (mode == MR_TILE_MODE_FP8_BLOCK && L->bits != 8)) {
    why = std::string(mode_name(mode)) + " fixes the element width";
    return false;
  }
  if (L->scale_block_rows <= 0) {
    why = "scaleBlockRows must be positive";
    return false;
  }
  if (block_scales(mode) ? L->scale_block_rows <= 1 : L->scale_block_rows != 1) {
    why = block_scales(mode) ? "a 2-D block-scale mode needs scaleBlockRows > 1"
                             : "one scale per row-group: scaleBlockRows must be 1";
    return false;
  }
  if (L->rows % L->scale_block_rows != 0) {
    why = "rows must be a multiple of scaleBlockRows";
    return false;
  }
  if (mode == MR_TILE_MODE_AFFINE && L->scale_dtype == MR_TILE_SCALE_E8M0) {
    why = "affine scales are a floating-point type; e8m0 is an MX encoding";
    return false;
  }
  if (L->cols % L->group_size != 0) {
    why = "cols " + str(L->cols) + " must be a multiple of the group size " + str(L->group_size);
    return false;
  }
  if (L->cols % (32 / L->bits) != 0) {
    why = "cols must fill whole 32-bit words";
    return false;
  }
  const int64_t groups_per_row = L->cols / L->group_size;
  const int64_t grid_rows = L->rows / L->scale_block_rows;
  L->packed_bytes = (int64_t)L->rows * L->cols * L->bits / 8;
  L->scale_bytes = grid_rows * groups_per_row * esz;
  L->bias_bytes = has_biases(mode) ? L->scale_bytes : 0;
  const bool padded = block_scales(mode);
  if (!padded) {
    if (L->packed_bytes % kTileAlign != 0) {
      why = "packed bytes per tile (" + str(L->packed_bytes) + ") must be a multiple of 16384";
      return false;
    }
    if (L->scale_bytes % kTileAlign != 0) {
      why = "scale bytes per tile (" + str(L->scale_bytes) + ") must be a multiple of 16384";
      return false;
    }
  }
  L->packed_region_bytes = align_up(L->packed_bytes, kTileAlign);
  L->scale_region_bytes = align_up(L->scale_bytes, kTileAlign);
  const int64_t bias_region = align_up(L->bias_bytes, kTileAlign);
  uint32_t flags = 0;
  if (has_biases(mode)) flags |= kFlagBiases;
  if (has_digests) flags |= kFlagDigests;
  if (L->scale_block_rows > 1) flags |= kFlag2D;
  if (padded) flags |= kFlagPadded;
  const bool v1 = mode == MR_TILE_MODE_MXFP4 && L->bits == 4 && L->group_size == 32 &&
                  L->scale_dtype == MR_TILE_SCALE_E8M0 && L->scale_block_rows == 1;
  int version;
  if (L->scale_block_rows != 1 || block_scales(mode)) version = 3;
  else if (!v1 || L->content_kind != MR_TILE_CONTENT_SYNTHETIC || flags != 0) version = 2;
  else version = 1;
  if (has_digests) {
    const int64_t capacity = (kTileHeaderBytes - digest_table_offset(version)) / kDigestBytes;
    if (tile_count > capacity) {
      why = "a 16384-byte header holds at most " + str(capacity) + " tile digests, not " +
            str(tile_count);
      return false;
    }
  }
  L->version = version;
  L->feature_flags = flags;
  L->tile_count = tile_count;
  L->scale_offset = L->packed_region_bytes;
  L->bias_offset = has_biases(mode) ? L->packed_region_bytes + L->scale_region_bytes : 0;
  L->tile_stride = L->packed_region_bytes + L->scale_region_bytes + bias_region;
  L->first_tile_offset = kTileHeaderBytes;
  L->total_bytes = L->first_tile_offset + tile_count * L->tile_stride;
  return true;
}

bool tile_decode_header(const unsigned char* h, mr_tile_layout* out,
                        std::vector<unsigned char>* digests, std::string& why) {
  if (memcmp(h, "MNRNTIL1", 8) != 0) {
    why = "not a tile container: bad magic";
    return false;
  }
  const uint32_t version = get_le<uint32_t>(h + 8);
  if (version < 1 || version > 3) {
    why = "tile container version " + str(version) + " is not supported (this build reads 1, 2, 3)";
    return false;
  }
  if (get_le<uint32_t>(h + 12) != (uint32_t)kTileHeaderBytes) {
    why = "header length is not 16384";
    return false;
  }
  mr_tile_layout L{};
  const uint32_t tile_count = get_le<uint32_t>(h + 16);
  L.rows = (int32_t)get_le<uint32_t>(h + 20);
  L.cols = (int32_t)get_le<uint32_t>(h + 24);
  L.group_size = (int32_t)get_le<uint32_t>(h + 28);
  const uint64_t packed = get_le<uint64_t>(h + 32), scales = get_le<uint64_t>(h + 40);
  const uint64_t scale_off = get_le<uint64_t>(h + 48), stride = get_le<uint64_t>(h + 56);
  const uint64_t first = get_le<uint64_t>(h + 64);
  L.seed = get_le<uint64_t>(h + 72);
  // version 1 has only these fields: 4-bit MXFP4, e8m0 scales, synthetic
  L.quant_mode = MR_TILE_MODE_MXFP4;
  L.bits = 4;
  L.content_kind = MR_TILE_CONTENT_SYNTHETIC;
  L.scale_dtype = MR_TILE_SCALE_E8M0;
  L.scale_block_rows = 1;
  uint32_t flags = 0;
  uint64_t bias_bytes = 0, bias_off = 0, packed_region = 0, scale_region = 0;
  bool has_regions = false;
  if (version >= 2) {
    L.quant_mode = (int32_t)get_le<uint32_t>(h + 80);
    if (L.quant_mode < 0 || L.quant_mode > MR_TILE_MODE_FP8_BLOCK) {
      why = "unknown quantization mode " + str(L.quant_mode);
      return false;
    }
    L.bits = (int32_t)get_le<uint32_t>(h + 84);
    L.content_kind = (int32_t)get_le<uint32_t>(h + 88);
    if (L.content_kind < 0 || L.content_kind > MR_TILE_CONTENT_CHECKPOINT) {
      why = "unknown content kind " + str(L.content_kind);
      return false;
    }
    flags = get_le<uint32_t>(h + 92);
    if (flags & ~kKnownFlags) {
      why = "feature flags include bits this build does not implement";
      return false;
    }
    bias_bytes = get_le<uint64_t>(h + 96);
    bias_off = get_le<uint64_t>(h + 104);
    const uint64_t digest_off = get_le<uint64_t>(h + 112);
    L.scale_dtype = (int32_t)get_le<uint32_t>(h + 120);
    if (scale_elem_bytes(L.scale_dtype) == 0) {
      why = "unknown scale element type " + str(L.scale_dtype);
      return false;
    }
    if (get_le<uint32_t>(h + 124) != 0) {
      why = "reserved header word is not zero";
      return false;
    }
    if (((flags & kFlagBiases) != 0) != has_biases(L.quant_mode)) {
      why = "the biases feature flag disagrees with the quantization mode";
      return false;
    }
    if (version >= 3) {
      L.scale_block_rows = (int32_t)get_le<uint32_t>(h + 128);
      packed_region = get_le<uint64_t>(h + 132);
      scale_region = get_le<uint64_t>(h + 140);
      has_regions = true;
      if (get_le<uint32_t>(h + 148) != 0 || get_le<uint64_t>(h + 152) != 0) {
        why = "reserved version-3 header words are not zero";
        return false;
      }
    } else if (flags & (kFlag2D | kFlagPadded)) {
      why = "a version-2 header sets a version-3 feature flag";
      return false;
    }
    const int table = digest_table_offset((int)version);
    if (flags & kFlagDigests) {
      if (digest_off != (uint64_t)table) {
        why = "digest table offset " + str((int64_t)digest_off) + " != " + str(table);
        return false;
      }
      const int64_t end = table + (int64_t)tile_count * kDigestBytes;
      if (end > kTileHeaderBytes) {
        why = "the digest table does not fit in the header";
        return false;
      }
      if (digests) digests->assign(h + table, h + end);
    } else if (digest_off != 0) {
      why = "a digest table offset is set but the feature flag is not";
      return false;
    }
  }
  // re-derive everything derivable and compare
  if (!tile_layout(&L, tile_count, (flags & kFlagDigests) != 0, why)) return false;
  if ((uint64_t)L.packed_bytes != packed || (uint64_t)L.scale_bytes != scales ||
      (uint64_t)L.scale_offset != scale_off || (uint64_t)L.tile_stride != stride ||
      (uint64_t)L.first_tile_offset != first || (uint64_t)L.bias_bytes != bias_bytes ||
      (uint64_t)L.bias_offset != bias_off) {
    why = "header fields contradict the geometry";
    return false;
  }
  if (has_regions && ((uint64_t)L.packed_region_bytes != packed_region ||
                      (uint64_t)L.scale_region_bytes != scale_region)) {
    why = "header sub-region sizes contradict the geometry";
    return false;
  }
  if ((uint32_t)L.version != version) {
    why = "file declares version " + str(version) + " but its contents are a version " +
          str(L.version) + " container";
    return false;
  }
  if (L.feature_flags != flags) {
    why = "feature flags contradict the geometry";
    return false;
  }
  *out = L;
  return true;
}

}  // namespace mr

namespace {

void set_msg(char* msg, size_t len, const std::string& s) {
  if (!msg || len == 0) return;
  const size_t n = s.size() < len - 1 ? s.size() : len - 1;
  memcpy(msg, s.data(), n);
  msg[n] = 0;
}

}  // namespace

extern "C" {

mr_status mr_sha256(const void* data, size_t bytes, uint8_t out[32]) {
  if ((!data && bytes) || !out) return MR_ERR_INVALID_ARGUMENT;
  mr::sha256(data, bytes, out);
  return MR_OK;
}

mr_status mr_tiles_layout_for(mr_tile_layout* lay, int64_t tile_count, int with_digests,
                              char* msg, size_t msg_len) {
  if (!lay) return MR_ERR_INVALID_ARGUMENT;
  std::string why;
  if (!mr::tile_layout(lay, tile_count, with_digests != 0, why)) {
    set_msg(msg, msg_len, why);
    return MR_ERR_UNSUPPORTED;
  }
  set_msg(msg, msg_len, "");
  return MR_OK;
}

mr_status mr_tiles_encode_header(const mr_tile_layout* lay, const uint8_t* digests,
                                  uint8_t* h, char* msg, size_t msg_len) {
  if (!lay || !h) return MR_ERR_INVALID_ARGUMENT;
  mr_tile_layout L = *lay;
  std::string why;
  const bool with = (lay->feature_flags & MR_TILE_FLAG_DIGESTS) != 0;
  if (with && !digests) {
    set_msg(msg, msg_len, "the layout records digests; pass them");
    return MR_ERR_INVALID_ARGUMENT;
  }
  if (!mr::tile_layout(&L, lay->tile_count, with, why)) {
    set_msg(msg, msg_len, why);
    return MR_ERR_UNSUPPORTED;
  }
  memset(h, 0, mr::kTileHeaderBytes);
  memcpy(h, "MNRNTIL1", 8);
  mr::put_le<uint32_t>(h + 8, (uint32_t)L.version);
  mr::put_le<uint32_t>(h + 12, (uint32_t)mr::kTileHeaderBytes);
  mr::put_le<uint32_t>(h + 16, (uint32_t)L.tile_count);
  mr::put_le<uint32_t>(h + 20, (uint32_t)L.rows);
  mr::put_le<uint32_t>(h + 24, (uint32_t)L.cols);
  mr::put_le<uint32_t>(h + 28, (uint32_t)L.group_size);
  mr::put_le<uint64_t>(h + 32, (uint64_t)L.packed_bytes);
  mr::put_le<uint64_t>(h + 40, (uint64_t)L.scale_bytes);
  mr::put_le<uint64_t>(h + 48, (uint64_t)L.scale_offset);
  mr::put_le<uint64_t>(h + 56, (uint64_t)L.tile_stride);
  mr::put_le<uint64_t>(h + 64, (uint64_t)L.first_tile_offset);
  mr::put_le<uint64_t>(h + 72, L.seed);
  if (L.version >= 2) {
    const int table = mr::digest_table_offset(L.version);
    mr::put_le<uint32_t>(h + 80, (uint32_t)L.quant_mode);
    mr::put_le<uint32_t>(h + 84, (uint32_t)L.bits);
    mr::put_le<uint32_t>(h + 88, (uint32_t)L.content_kind);
    mr::put_le<uint32_t>(h + 92, L.feature_flags);
    mr::put_le<uint64_t>(h + 96, (uint64_t)L.bias_bytes);
    mr::put_le<uint64_t>(h + 104, (uint64_t)L.bias_offset);
    mr::put_le<uint64_t>(h + 112, with ? (uint64_t)table : 0);
    mr::put_le<uint32_t>(h + 120, (uint32_t)L.scale_dtype);
    if (L.version >= 3) {
      mr::put_le<uint32_t>(h + 128, (uint32_t)L.scale_block_rows);
      mr::put_le<uint64_t>(h + 132, (uint64_t)L.packed_region_bytes);
      mr::put_le<uint64_t>(h + 140, (uint64_t)L.scale_region_bytes);
    }
    if (with) memcpy(h + table, digests, (size_t)L.tile_count * mr::kDigestBytes);
  }
  set_msg(msg, msg_len, "");
  return MR_OK;
}

mr_status mr_tiles_open(const char* path, int verify_digests, mr_tiles** out, char* msg,
                        size_t msg_len) {
  if (!path || !out) return MR_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    set_msg(msg, msg_len, std::string("open '") + path + "': " + strerror(errno));
    return MR_ERR_IO;
  }
  std::vector<unsigned char> h(mr::kTileHeaderBytes);
  size_t got = 0;
  while (got < h.size()) {
    const ssize_t r = ::pread(fd, h.data() + got, h.size() - got, (off_t)got);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) break;
    got += (size_t)r;
  }
  if (got < h.size()) {
    ::close(fd);
    set_msg(msg, msg_len, std::string("tile container '") + path + "' is truncated: header needs " +
                              mr::str(mr::kTileHeaderBytes) + " bytes, read " + mr::str(got));
    return MR_ERR_IO;
  }
  mr_tiles* t = new mr_tiles;
  t->fd = fd;
  t->path = path;
  t->verify = verify_digests != 0;
  std::string why;
  if (!mr::tile_decode_header(h.data(), &t->layout, &t->digests, why)) {
    mr_tiles_close(t);
    set_msg(msg, msg_len, std::string("tile container '") + path + "': " + why);
    return MR_ERR_INVALID_ARGUMENT;
  }
  struct stat stt;
  if (fstat(fd, &stt) != 0 || (int64_t)stt.st_size < t->layout.total_bytes) {
    const int64_t have = fstat(fd, &stt) == 0 ? (int64_t)stt.st_size : -1;
    mr_tiles_close(t);
    set_msg(msg, msg_len, std::string("tile container '") + path +
                              "' is truncated: header describes " + mr::str(t->layout.total_bytes) +
                              " bytes, file is " + mr::str(have));
    return MR_ERR_IO;
  }
  set_msg(msg, msg_len, "");
  *out = t;
  return MR_OK;
}

mr_status mr_tiles_close(mr_tiles* t) {
  if (!t) return MR_OK;
  if (t->fd >= 0) ::close(t->fd);
  delete t;
  return MR_OK;
}

mr_status mr_tiles_get_layout(const mr_tiles* t, mr_tile_layout* out) {
  if (!t || !out) return MR_ERR_INVALID_ARGUMENT;
  *out = t->layout;
  return MR_OK;
}

mr_status mr_tiles_read(mr_tiles* t, int64_t tile, void* dst, size_t dst_bytes, char* msg,
                        size_t msg_len) {
  if (!t || !dst) return MR_ERR_INVALID_ARGUMENT;
  const mr_tile_layout& L = t->layout;
  if (tile < 0 || tile >= L.tile_count) {
    set_msg(msg, msg_len, "tile " + mr::str(tile) + " requested from a container of " +
                              mr::str(L.tile_count) + " tiles");
    return MR_ERR_INVALID_ARGUMENT;
  }
  if ((int64_t)dst_bytes < L.tile_stride) {
    set_msg(msg, msg_len, "a tile is " + mr::str(L.tile_stride) + " bytes; the buffer holds " +
                              mr::str((int64_t)dst_bytes));
    return MR_ERR_INVALID_ARGUMENT;
  }
  const off_t base = (off_t)(L.first_tile_offset + tile * L.tile_stride);
  unsigned char* p = static_cast<unsigned char*>(dst);
  int64_t got = 0;
  while (got < L.tile_stride) {
    const ssize_t r = ::pread(t->fd, p + got, (size_t)(L.tile_stride - got), base + (off_t)got);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) {
      set_msg(msg, msg_len, "pread of tile " + mr::str(tile) + " of '" + t->path + "' " +
                                (r < 0 ? std::string("failed: ") + strerror(errno)
                                       : std::string("ended early")));
      return MR_ERR_IO;
    }
    got += r;
  }
  if (t->verify && !t->digests.empty()) {
    unsigned char d[32];
    mr::sha256(dst, (size_t)L.tile_stride, d);
    if (memcmp(d, t->digests.data() + tile * 32, 32) != 0) {
      set_msg(msg, msg_len, "tile " + mr::str(tile) + " of '" + t->path +
                                "' fails its recorded SHA-256");
      return MR_ERR_INTEGRITY;
    }
  }
  set_msg(msg, msg_len, "");
  return MR_OK;
}

}  // extern "C"
