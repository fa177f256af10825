// mann.cu -- read-only loader of the reference's index files ("MANN", format
// versions 1-3 of IndexSerializer.save / saveMmapCompatible,
// Sources/MetalANNSCore/IndexSerializer.swift:11-137, read as
// IndexSerializer.load :141-316 and MmapIndexLoader.load,
// Sources/MetalANNSCore/MmapIndexLoader.swift:38-200 do) into a device corpus.
//
// Layout (little-endian u32 fields): "MANN", version, nodeCount, degree, dim,
// metric code, storage type (version >= 2; 0 fp32, 1 fp16, 2 binary); then
// the vectors (nodeCount x dim), the adjacency (nodeCount x degree u32) and the
// edge distances (nodeCount x degree f32) -- in version 3 each section starts
// on a page boundary of the writer's page size -- then a u32 byte count, the
// JSON IDMap and a u32 entry point.  The vectors are the corpus of the exact
// search; the graph sections and the IDMap stay on the host side.

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "internal.h"
#include "mans_cuda.h"

namespace mans {
namespace {

struct Mapped {
  const uint8_t* p = nullptr;
  size_t len = 0;
  int fd = -1;
  ~Mapped() {
    if (p) munmap(const_cast<uint8_t*>(p), len);
    if (fd >= 0) close(fd);
  }
};

int32_t map_file(const char* path, Mapped& m) {
  m.fd = open(path, O_RDONLY);
  if (m.fd < 0) return fail(MANS_ERR_CORRUPT, "cannot open the index file");
  struct stat st;
  if (fstat(m.fd, &st) != 0 || st.st_size <= 0) return fail(MANS_ERR_CORRUPT, "File is too small");
  m.len = static_cast<size_t>(st.st_size);
  void* p = mmap(nullptr, m.len, PROT_READ, MAP_PRIVATE, m.fd, 0);
  if (p == MAP_FAILED) return fail(MANS_ERR_CORRUPT, "cannot map the index file");
  m.p = static_cast<const uint8_t*>(p);
  return MANS_OK;
}

uint32_t rd32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
         (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24);
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
  if (a != 0 && b > UINT64_MAX / a) return false;
  *out = a * b;
  return true;
}

uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Parses the header and locates every section.  A version-3 file carries no
// record of its writer's page size (16 KiB on Apple silicon, 4 KiB on most
// Linux hosts), so each candidate is tried and the one whose trailer -- u32
// length, JSON object, u32 entry point -- ends exactly at the end of the file
// is taken.
int32_t parse(const uint8_t* p, size_t len, mans_mann_info* info) {
  std::memset(info, 0, sizeof *info);
  if (len < 24) return fail(MANS_ERR_CORRUPT, "File is too small");
  if (std::memcmp(p, "MANN", 4) != 0) return fail(MANS_ERR_CORRUPT, "Invalid file magic");
  info->version = rd32(p + 4);
  if (info->version < 1 || info->version > 3)
    return fail(MANS_ERR_CORRUPT, "Unsupported file version");
  info->count = rd32(p + 8);
  info->degree = rd32(p + 12);
  info->dim = rd32(p + 16);
  info->metric = rd32(p + 20);
  uint64_t cursor = 24;
  if (info->version >= 2) {
    if (len < 28) return fail(MANS_ERR_CORRUPT, "File is too small");
    info->storage = rd32(p + 24);
    cursor = 28;
  }
  if (info->metric > 3) return fail(MANS_ERR_CORRUPT, "Unsupported metric code");
  if (info->storage > 2) return fail(MANS_ERR_CORRUPT, "Unsupported storage type");
  if (info->count == 0) return fail(MANS_ERR_CORRUPT, "Node count must be greater than zero");
  if (info->degree == 0) return fail(MANS_ERR_CORRUPT, "Degree must be greater than zero");
  if (info->dim == 0) return fail(MANS_ERR_CORRUPT, "Dimension must be greater than zero");
  uint64_t vbytes = 0, ebytes = 0, edges = 0;
  if (info->storage == 2) {
    if (info->dim % 8 != 0) return fail(MANS_ERR_CORRUPT, "Binary index has dim not divisible by 8");
    vbytes = static_cast<uint64_t>(info->count) * (info->dim / 8);
  } else if (!mul_ok(static_cast<uint64_t>(info->count) * info->dim,
                     info->storage == 1 ? 2 : 4, &vbytes)) {
    return fail(MANS_ERR_CORRUPT, "Integer overflow while computing serialized sizes");
  }
  if (!mul_ok(info->count, info->degree, &edges) || !mul_ok(edges, 4, &ebytes))
    return fail(MANS_ERR_CORRUPT, "Integer overflow while computing serialized sizes");
  info->vector_bytes = vbytes;
  auto trailer_at = [&](uint64_t off) -> bool {
    if (off + 4 > len) return false;
    const uint64_t n = rd32(p + off);
    if (off + 4 + n + 4 != len) return false;
    return n == 0 || p[off + 4] == '{';
  };
  if (info->version == 3) {
    const uint32_t pages[] = {16384, 4096, 65536, 8192};
    for (uint32_t pg : pages) {
      const uint64_t v0 = align_up(cursor, pg);
      const uint64_t a0 = align_up(v0 + vbytes, pg);
      const uint64_t d0 = align_up(a0 + ebytes, pg);
      const uint64_t t0 = align_up(d0 + ebytes, pg);
      if (t0 + 4 <= len && trailer_at(t0)) {
        info->page_size = pg;
        info->vector_offset = v0;
        info->adjacency_offset = a0;
        info->distance_offset = d0;
        info->idmap_offset = t0 + 4;
        info->idmap_bytes = rd32(p + t0);
        info->entry_point = rd32(p + t0 + 4 + info->idmap_bytes);
        break;
      }
    }
    if (info->page_size == 0) return fail(MANS_ERR_CORRUPT, "Mmap sections are truncated");
  } else {
    info->vector_offset = cursor;
    info->adjacency_offset = cursor + vbytes;
    info->distance_offset = info->adjacency_offset + ebytes;
    const uint64_t t0 = info->distance_offset + ebytes;
    if (t0 + 4 > len) return fail(MANS_ERR_CORRUPT, "Corrupt or truncated body");
    info->idmap_bytes = rd32(p + t0);
    if (t0 + 4 + info->idmap_bytes + 4 > len)
      return fail(MANS_ERR_CORRUPT, "Truncated or invalid IDMap payload");
    info->idmap_offset = t0 + 4;
    info->entry_point = rd32(p + t0 + 4 + info->idmap_bytes);
  }
  if (info->entry_point >= info->count) return fail(MANS_ERR_CORRUPT, "Entry point is out of bounds");
  return MANS_OK;
}

// IEEE binary16 -> binary32 (exact: every half value is a float value)
float half_to_float(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: normalise
      exp = 127 - 15 + 1;
      while ((man & 0x400u) == 0) {
        man <<= 1;
        --exp;
      }
      man &= 0x3FFu;
      bits = sign | (exp << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp - 15 + 127) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

}  // namespace
}  // namespace mans

extern "C" {

int32_t mans_mann_read_info(const char* path, mans_mann_info* out) {
  using namespace mans;
  if (!path || !out) return fail(MANS_ERR_INVALID, "null path or output");
  Mapped m;
  int32_t rc = map_file(path, m);
  if (rc != MANS_OK) return rc;
  return parse(m.p, m.len, out);
}

int32_t mans_corpus_load_mann(mans_ctx* ctx, const char* path, int32_t shard_index,
                              int32_t shard_count, mans_corpus** out_corpus) {
  using namespace mans;
  if (!ctx || !path || !out_corpus) return fail(MANS_ERR_INVALID, "null context, path or output");
  *out_corpus = nullptr;
  if (shard_count < 1 || shard_index < 0 || shard_index >= shard_count)
    return fail(MANS_ERR_INVALID, "bad shard index / count");
  Mapped m;
  int32_t rc = map_file(path, m);
  if (rc != MANS_OK) return rc;
  mans_mann_info info;
  if ((rc = parse(m.p, m.len, &info)) != MANS_OK) return rc;
  if (info.storage == 2)
    return fail(MANS_ERR_SEARCH, "binary (Hamming) storage has no float corpus");
  // rows of this shard: the first count % shard_count shards hold one more
  const int64_t n = info.count, dim = info.dim;
  const int64_t base = n / shard_count, extra = n % shard_count;
  const int64_t r0 = shard_index * base + std::min<int64_t>(shard_index, extra);
  const int64_t rows = base + (shard_index < extra ? 1 : 0);
  const uint8_t* vec = m.p + info.vector_offset;
  if (info.storage == 0) {
    // fp32 rows straight from the mapped pages
    return corpus_create_any(ctx, reinterpret_cast<const float*>(vec) + r0 * dim, rows, dim,
                             static_cast<uint32_t>(r0), out_corpus);
  }
  std::vector<float> wide(static_cast<size_t>(std::max<int64_t>(rows, 1)) * dim);
  const uint8_t* src = vec + static_cast<size_t>(r0) * dim * 2;
  for (size_t i = 0; i < static_cast<size_t>(rows) * dim; ++i) {
    uint16_t h;
    std::memcpy(&h, src + 2 * i, 2);
    wide[i] = half_to_float(h);
  }
  return corpus_create_any(ctx, wide.data(), rows, dim, static_cast<uint32_t>(r0), out_corpus);
}

}  // extern "C"
