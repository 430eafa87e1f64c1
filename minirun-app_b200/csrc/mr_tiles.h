// mr_tiles.h — the MNRNTIL1 quantized tile container (host side): header
// decoding with the reference reader's validation rules, whole-tile reads,
// per-tile SHA-256 checks. The format and its rules follow
// Sources/StorageCore/Container/QuantizedTileContainer.swift (layout:
// :441-580, header encoding :739-784, decoding and validation :811-1001,
// digest check :1153-1181).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "minirun_moe.h"

namespace mr {

constexpr int kTileAlign = 16384;  // every tile and sub-region starts on this boundary
constexpr int kTileHeaderBytes = kTileAlign;

// Computes the layout of a geometry the way a writer must lay it out and a
// reader re-derives it; false (with `why`) for geometries the format rejects.
// `lay` carries the geometry in and the derived fields out.
bool tile_layout(mr_tile_layout* lay, int64_t tile_count, bool has_digests, std::string& why);

// Decodes and validates a 16 KiB header; digests (32 bytes per tile) are
// copied out when the file carries them.
bool tile_decode_header(const unsigned char* h, mr_tile_layout* lay,
                        std::vector<unsigned char>* digests, std::string& why);

// FIPS 180-4 SHA-256.
void sha256(const void* data, size_t n, unsigned char out[32]);

}  // namespace mr

// An open container: the descriptor, its layout and digest table.
struct mr_tiles {
  int fd = -1;
  std::string path;
  mr_tile_layout layout{};
  std::vector<unsigned char> digests;  // tile_count * 32, or empty
  bool verify = false;
};
