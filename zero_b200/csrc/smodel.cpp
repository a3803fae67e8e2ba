// smodel.cpp — the SilicatePack `.smodel` container reader (host code).
//
// Maps a native `.smodel` file read-only and validates it with the rules of
// the reference's loader (kernel/src/model_loader.rs):
//   * header (smodel_info, model_loader.rs:599-661): 128 bytes
//     "<4sIIQQQQII32s" = magic SILM, version 1 or 2 (v2: row-interleaved
//     dtypes allowed), header_len 128, manifest offset/len, payload
//     offset/len, payload kind (1 GGUF-compat, 2 native), flags (bit 0: the
//     payload is 2 MiB aligned), payload SHA-256; the manifest and the payload
//     inside the file, the manifest before the payload;
//   * native index (smodel_native_summary / smodel_native_tensor_index,
//     model_loader.rs:256-597): "SIDX" v1, a 128-byte header carrying the
//     model fields, tensor_count <= 10 000 entries of 104 bytes
//     ("<IIII8Q3Q": name offset, name length, dtype id, rank, shape[8],
//     payload offset, byte length, elements), then the names blob; every name
//     valid UTF-8 inside the blob, every tensor inside the payload, the
//     row-interleaved dtypes (100 Q4_0X4, 101 Q8_0X4) only on rank-2 tensors
//     whose first dimension (output rows; SIDX keeps the HF order) is a
//     multiple of 4.
// Tensor offsets are relative to the payload.  Error classes map onto the
// loader's LoadError: MagicMismatch, UnsupportedFormat, InvalidContainer.
// zgpu_smodel_register uploads the matmul tensors keyed by their mapped
// addresses, the layout registry weight_layout::register keys by
// (weight_layout.rs:11-19, model_loader.rs:560-566).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/zgpu.h"

namespace {

constexpr uint32_t kMagicSilm = 0x4D4C4953u;   // "SILM"
constexpr uint32_t kMagicSidx = 0x58444953u;   // "SIDX"
constexpr uint64_t kHeaderSize = 128, kIndexHeaderSize = 128, kEntrySize = 104;
constexpr uint64_t kMaxTensors = 10000;
constexpr uint64_t kPayloadAlignment = 2ull << 20;

thread_local std::string g_error;

uint32_t rd32(const uint8_t *p) {
  uint32_t v;
  std::memcpy(&v, p, 4);
  return v;
}
uint64_t rd64(const uint8_t *p) {
  uint64_t v;
  std::memcpy(&v, p, 8);
  return v;
}
float rdf(const uint8_t *p) {
  float v;
  std::memcpy(&v, p, 4);
  return v;
}

// SIDX dtype ids the packer emits (silicatepack.py NATIVE_DTYPE_IDS): the
// GGML ids, plus the .smodel-v2 row-interleaved 100 / 101.
bool known_dtype(uint32_t d) {
  switch (d) {
    case 0: case 1: case 2: case 3: case 6: case 7: case 8: case 9: case 10: case 11: case 12:
    case 13: case 14: case 15: case 20: case 24: case 25: case 26: case 27: case 28: case 30:
    case 100: case 101:
      return true;
    default:
      return false;
  }
}

bool valid_utf8(const uint8_t *s, uint64_t n) {
  uint64_t i = 0;
  while (i < n) {
    const uint8_t c = s[i];
    uint32_t len, cp;
    if (c < 0x80) {
      ++i;
      continue;
    } else if ((c & 0xE0) == 0xC0) {
      len = 2;
      cp = c & 0x1F;
    } else if ((c & 0xF0) == 0xE0) {
      len = 3;
      cp = c & 0x0F;
    } else if ((c & 0xF8) == 0xF0) {
      len = 4;
      cp = c & 0x07;
    } else {
      return false;
    }
    if (i + len > n) return false;
    for (uint32_t k = 1; k < len; ++k) {
      if ((s[i + k] & 0xC0) != 0x80) return false;
      cp = (cp << 6) | (s[i + k] & 0x3F);
    }
    if ((len == 2 && cp < 0x80) || (len == 3 && cp < 0x800) || (len == 4 && cp < 0x10000) || cp > 0x10FFFF ||
        (cp >= 0xD800 && cp <= 0xDFFF))
      return false;
    i += len;
  }
  return true;
}

zgpu_status fail(zgpu_status s, const std::string &msg) {
  g_error = msg;
  return s;
}

}  // namespace

struct zgpu_smodel {
  const uint8_t *base = nullptr;
  size_t size = 0;
  zgpu_smodel_info info = {};
  std::vector<zgpu_smodel_tensor> tensors;
  std::vector<std::string> names;
};

extern "C" {

const char *zgpu_smodel_error(void) { return g_error.c_str(); }

void zgpu_smodel_close(zgpu_smodel *m) {
  if (!m) return;
  if (m->base) munmap(const_cast<uint8_t *>(m->base), m->size);
  delete m;
}

zgpu_status zgpu_smodel_open(const char *path, zgpu_smodel **out) {
  if (!path || !out) return ZGPU_ERR_INVALID_ARG;
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(ZGPU_ERR_MODEL_IO, std::string("cannot open ") + path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    return fail(ZGPU_ERR_MODEL_IO, "cannot stat the model file");
  }
  const size_t size = static_cast<size_t>(st.st_size);
  void *map = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (map == MAP_FAILED) return fail(ZGPU_ERR_MODEL_IO, "cannot map the model file");
  zgpu_smodel *m = new (std::nothrow) zgpu_smodel();
  if (!m) {
    munmap(map, size);
    return ZGPU_ERR_OUT_OF_MEMORY;
  }
  m->base = static_cast<const uint8_t *>(map);
  m->size = size;
  auto reject = [&](zgpu_status s, const std::string &msg) {
    zgpu_smodel_close(m);
    return fail(s, msg);
  };
  const uint8_t *b = m->base;
  // ---- container header (smodel_info)
  if (size < kHeaderSize) return reject(ZGPU_ERR_MODEL_INVALID, "file shorter than the 128-byte header");
  if (rd32(b) != kMagicSilm) return reject(ZGPU_ERR_MODEL_MAGIC, "not a SilicatePack container (magic)");
  zgpu_smodel_info &in = m->info;
  in.version = rd32(b + 4);
  if (in.version != 1 && in.version != 2) return reject(ZGPU_ERR_MODEL_UNSUPPORTED, "container version not 1 or 2");
  const uint64_t header_len = rd32(b + 8);
  in.manifest_offset = rd64(b + 12);
  in.manifest_len = rd64(b + 20);
  in.payload_offset = rd64(b + 28);
  in.payload_len = rd64(b + 36);
  in.payload_kind = rd32(b + 44);
  in.flags = rd32(b + 48);
  if (header_len != kHeaderSize) return reject(ZGPU_ERR_MODEL_UNSUPPORTED, "header length not 128");
  if (in.payload_kind != 1 && in.payload_kind != 2) return reject(ZGPU_ERR_MODEL_UNSUPPORTED, "unknown payload kind");
  if (in.manifest_len == 0) return reject(ZGPU_ERR_MODEL_INVALID, "empty manifest");
  const uint64_t manifest_end = in.manifest_offset + in.manifest_len, payload_end = in.payload_offset + in.payload_len;
  if (manifest_end < in.manifest_offset || payload_end < in.payload_offset || in.manifest_offset < header_len ||
      manifest_end > in.payload_offset || in.payload_offset < header_len || payload_end > size || in.payload_len < 4)
    return reject(ZGPU_ERR_MODEL_INVALID, "manifest / payload outside the file");
  if ((in.flags & 1u) && in.payload_offset % kPayloadAlignment)
    return reject(ZGPU_ERR_MODEL_INVALID, "payload flagged 2 MiB aligned but is not");
  if (in.payload_kind != 2)
    return reject(ZGPU_ERR_MODEL_UNSUPPORTED, "GGUF-compat payload: only native payloads are read");
  if (in.payload_len < kIndexHeaderSize) return reject(ZGPU_ERR_MODEL_INVALID, "payload shorter than the SIDX header");
  // ---- native index (smodel_native_summary / smodel_native_tensor_index)
  const uint8_t *p = b + in.payload_offset;
  const uint64_t plen = in.payload_len;
  if (rd32(p) != kMagicSidx || rd32(p + 4) != 1 || rd32(p + 8) != kIndexHeaderSize)
    return reject(ZGPU_ERR_MODEL_UNSUPPORTED, "not a SIDX v1 index");
  const uint64_t count = rd32(p + 12);
  if (count > kMaxTensors) return reject(ZGPU_ERR_MODEL_INVALID, "tensor count above 10000");
  const uint64_t entry_size = rd32(p + 16), names_offset = rd32(p + 20), names_len = rd32(p + 24);
  if (entry_size != kEntrySize) return reject(ZGPU_ERR_MODEL_UNSUPPORTED, "SIDX entry size not 104");
  const uint64_t entries_end = kIndexHeaderSize + count * entry_size, names_end = names_offset + names_len;
  if (entries_end > plen || names_offset < entries_end || names_end > plen)
    return reject(ZGPU_ERR_MODEL_INVALID, "SIDX entries / names outside the payload");
  in.tensor_count = static_cast<uint32_t>(count);
  in.data_base = rd64(p + 28);
  in.architecture_id = rd32(p + 36);
  in.block_count = rd32(p + 40);
  in.context_length = rd32(p + 44);
  in.embedding_length = rd32(p + 48);
  in.feed_forward_length = rd32(p + 52);
  in.head_count = rd32(p + 56);
  in.head_count_kv = rd32(p + 60);
  in.key_length = rd32(p + 64);
  in.value_length = rd32(p + 68);
  in.rope_freq_base = rdf(p + 72);
  in.layer_norm_rms_epsilon = rdf(p + 76);
  in.vocab_size = rd32(p + 80);
  in.eos_token_id = rd32(p + 84);
  in.expert_count = rd32(p + 88);
  in.expert_used_count = rd32(p + 92);
  in.expert_shared_count = rd32(p + 96);
  in.expert_feed_forward_length = rd32(p + 100);
  in.kv_lora_rank = rd32(p + 104);
  in.q_lora_rank = rd32(p + 108);
  in.qk_nope_head_dim = rd32(p + 112);
  in.qk_rope_head_dim = rd32(p + 116);
  in.v_head_dim = rd32(p + 120);
  in.expert_weights_scale = rdf(p + 124);
  const uint8_t *names = p + names_offset;
  m->tensors.resize(count);
  m->names.resize(count);
  for (uint64_t i = 0; i < count; ++i) {
    const uint8_t *e = p + kIndexHeaderSize + i * entry_size;
    const uint64_t name_off = rd32(e), name_len = rd32(e + 4);
    zgpu_smodel_tensor &t = m->tensors[i];
    t.dtype = rd32(e + 8);
    t.rank = rd32(e + 12);
    if (t.rank > 8) return reject(ZGPU_ERR_MODEL_INVALID, "tensor rank above 8");
    if (name_off + name_len < name_off || name_off + name_len > names_len || !valid_utf8(names + name_off, name_len))
      return reject(ZGPU_ERR_MODEL_INVALID, "tensor name outside the names blob or not UTF-8");
    m->names[i].assign(reinterpret_cast<const char *>(names + name_off), name_len);
    if (!known_dtype(t.dtype)) return reject(ZGPU_ERR_MODEL_UNSUPPORTED, "unknown tensor dtype in " + m->names[i]);
    for (uint32_t d = 0; d < 8; ++d) t.shape[d] = rd64(e + 16 + 8 * d);
    t.payload_offset = rd64(e + 80);
    t.byte_len = rd64(e + 88);
    t.elements = rd64(e + 96);
    if (t.payload_offset + t.byte_len < t.payload_offset || t.payload_offset + t.byte_len > plen)
      return reject(ZGPU_ERR_MODEL_INVALID, "tensor " + m->names[i] + " outside the payload");
    if ((t.dtype == 100 || t.dtype == 101) && (t.rank != 2 || t.shape[0] % 4))
      return reject(ZGPU_ERR_MODEL_INVALID, "interleaved tensor " + m->names[i] + " with rows not a multiple of 4");
    t.data = p + t.payload_offset;
  }
  for (uint64_t i = 0; i < count; ++i) m->tensors[i].name = m->names[i].c_str();
  *out = m;
  return ZGPU_OK;
}

zgpu_status zgpu_smodel_info_get(const zgpu_smodel *m, zgpu_smodel_info *out) {
  if (!m || !out) return ZGPU_ERR_INVALID_ARG;
  *out = m->info;
  return ZGPU_OK;
}

zgpu_status zgpu_smodel_manifest(const zgpu_smodel *m, const char **json, uint64_t *len) {
  if (!m || !json || !len) return ZGPU_ERR_INVALID_ARG;
  *json = reinterpret_cast<const char *>(m->base + m->info.manifest_offset);
  *len = m->info.manifest_len;
  return ZGPU_OK;
}

zgpu_status zgpu_smodel_tensor_at(const zgpu_smodel *m, uint32_t i, zgpu_smodel_tensor *out) {
  if (!m || !out || i >= m->tensors.size()) return ZGPU_ERR_INVALID_ARG;
  *out = m->tensors[i];
  return ZGPU_OK;
}

zgpu_status zgpu_smodel_find(const zgpu_smodel *m, const char *name, zgpu_smodel_tensor *out) {
  if (!m || !name || !out) return ZGPU_ERR_INVALID_ARG;
  for (size_t i = 0; i < m->tensors.size(); ++i)
    if (m->names[i] == name) {
      *out = m->tensors[i];
      return ZGPU_OK;
    }
  return fail(ZGPU_ERR_UNREGISTERED_WEIGHT, std::string("no tensor named ") + name);
}

zgpu_status zgpu_smodel_register(zgpu_ctx *ctx, const zgpu_smodel *m, uint32_t *registered) {
  if (!ctx || !m) return ZGPU_ERR_INVALID_ARG;
  uint32_t n = 0;
  for (const zgpu_smodel_tensor &t : m->tensors) {
    const bool matmul_dtype = t.dtype == ZGPU_F32 || t.dtype == ZGPU_Q4_0 || t.dtype == ZGPU_Q8_0 ||
                              t.dtype == ZGPU_Q4_0X4 || t.dtype == ZGPU_Q8_0X4;
    if (t.rank != 2 || !matmul_dtype) continue;
    const zgpu_status s = zgpu_register_weights(ctx, t.data, t.byte_len, t.dtype, t.shape[0], t.shape[1]);
    if (s != ZGPU_OK) return s;
    ++n;
  }
  if (registered) *registered = n;
  return ZGPU_OK;
}

}  // extern "C"
