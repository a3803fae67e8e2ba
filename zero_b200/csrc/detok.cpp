// detok.cpp — token ids -> bytes for streaming output (the kernel's
// detokenizer, kernel/src/detokenizer.rs:110-273): a vocabulary of byte
// strings with a u32 offset table of vocab_size + 1 entries, installed once
// (install_runtime_vocab, :208-256, copies both tables) and read by id.
// Host code: the lookup is a table read per generated token.
#include <cstring>
#include <new>
#include <vector>

#include "../../include/zgpu.h"

struct zgpu_detok {
  std::vector<uint8_t> bytes;
  std::vector<uint32_t> offsets;   // vocab + 1 entries
  uint32_t vocab = 0;
};

namespace {

// decode_token (detokenizer.rs:110-131, runtime path :166-205): an id past
// the vocabulary, or an entry whose offsets run backwards or past the byte
// table, decodes to nothing.
void token_slice(const zgpu_detok *d, uint32_t id, const uint8_t **p, uint64_t *n) {
  *p = d->bytes.data();
  *n = 0;
  if (id >= d->vocab) return;
  const uint32_t start = d->offsets[id], end = d->offsets[id + 1];
  if (end > d->bytes.size() || start > end) return;
  *p = d->bytes.data() + start;
  *n = end - start;
}

}  // namespace

extern "C" {

zgpu_status zgpu_detok_create(const void *bytes, uint64_t n_bytes, const uint32_t *offsets, uint32_t vocab_size,
                              zgpu_detok **out) {
  if (!out || !offsets || vocab_size == 0 || (n_bytes && !bytes)) return ZGPU_ERR_INVALID_ARG;
  *out = nullptr;
  zgpu_detok *d = new (std::nothrow) zgpu_detok();
  if (!d) return ZGPU_ERR_OUT_OF_MEMORY;
  try {
    d->bytes.assign(static_cast<const uint8_t *>(bytes), static_cast<const uint8_t *>(bytes) + n_bytes);
    d->offsets.assign(offsets, offsets + static_cast<size_t>(vocab_size) + 1);
  } catch (...) {
    delete d;
    return ZGPU_ERR_OUT_OF_MEMORY;
  }
  d->vocab = vocab_size;
  *out = d;
  return ZGPU_OK;
}

void zgpu_detok_destroy(zgpu_detok *d) { delete d; }

uint32_t zgpu_detok_vocab_size(const zgpu_detok *d) { return d ? d->vocab : 0; }

zgpu_status zgpu_detok_token(const zgpu_detok *d, uint32_t id, const uint8_t **bytes_out, uint64_t *len_out) {
  if (!d || !bytes_out || !len_out) return ZGPU_ERR_INVALID_ARG;
  token_slice(d, id, bytes_out, len_out);
  return ZGPU_OK;
}

zgpu_status zgpu_detok_decode(const zgpu_detok *d, const uint32_t *ids, uint64_t n, uint8_t *out, uint64_t cap,
                              uint64_t *written) {
  if (!d || (n && !ids) || !written) return ZGPU_ERR_INVALID_ARG;
  uint64_t total = 0;
  for (uint64_t i = 0; i < n; ++i) {
    const uint8_t *p;
    uint64_t len;
    token_slice(d, ids[i], &p, &len);
    total += len;
  }
  *written = total;
  if (total > cap || (total && !out)) return ZGPU_ERR_INVALID_ARG;   // *written holds the size needed
  uint64_t at = 0;
  for (uint64_t i = 0; i < n; ++i) {
    const uint8_t *p;
    uint64_t len;
    token_slice(d, ids[i], &p, &len);
    if (len) std::memcpy(out + at, p, len);
    at += len;
  }
  return ZGPU_OK;
}

}  // extern "C"
