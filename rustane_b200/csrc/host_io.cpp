// Host-side training I/O of the engine, native: the token data files and the
// sampling positions of the training loop (crates/engine/src/data.rs:11-95,
// bin/train.rs:116-140, 285-290), val bits-per-byte (data.rs:67-89), and the
// RSTK checkpoint format (bin/train.rs:165-202) with a reader and an optional
// optimizer-state extension.  No CUDA: these run on the host only.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "rustane_cuda.h"

struct rt_tokens {
  const uint16_t* data = nullptr;
  size_t bytes = 0;
  int64_t n = 0;
};

namespace {

// LayerWeights field order of the checkpoint (bin/train.rs:187-191) with element counts.
void layer_sizes(const rt_model_config& c, int64_t (&n)[9]) {
  const int64_t D = c.dim, Q = c.q_dim, KV = c.kv_dim, H = c.hidden;
  const int64_t s[9] = {D * Q, D * KV, D * KV, Q * D, D * H, D * H, D * H, D, D};
  for (int i = 0; i < 9; ++i) n[i] = s[i];
}
float* layer_field(const rt_layer_ptrs& l, int i) {
  float* const f[9] = {l.wq, l.wk, l.wv, l.wo, l.w1, l.w3, l.w2, l.gamma1, l.gamma2};
  return f[i];
}

bool write_model(FILE* f, const rt_model_config& c, const rt_model_ptrs& w) {
  const int64_t D = c.dim, V = c.vocab;
  if (fwrite(w.embed, sizeof(float), V * D, f) != size_t(V * D)) return false;
  if (fwrite(w.gamma_final, sizeof(float), D, f) != size_t(D)) return false;
  int64_t n[9];
  layer_sizes(c, n);
  for (int l = 0; l < c.nlayers; ++l)
    for (int i = 0; i < 9; ++i)
      if (fwrite(layer_field(w.layers[l], i), sizeof(float), n[i], f) != size_t(n[i])) return false;
  return true;
}
bool read_model(FILE* f, const rt_model_config& c, const rt_model_ptrs& w) {
  const int64_t D = c.dim, V = c.vocab;
  if (fread(w.embed, sizeof(float), V * D, f) != size_t(V * D)) return false;
  if (fread(w.gamma_final, sizeof(float), D, f) != size_t(D)) return false;
  int64_t n[9];
  layer_sizes(c, n);
  for (int l = 0; l < c.nlayers; ++l)
    for (int i = 0; i < 9; ++i)
      if (fread(layer_field(w.layers[l], i), sizeof(float), n[i], f) != size_t(n[i])) return false;
  return true;
}

void put_u32(unsigned char* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = static_cast<unsigned char>(v >> (8 * i));
}
uint32_t get_u32(const unsigned char* p) {
  return uint32_t(p[0]) | uint32_t(p[1]) << 8 | uint32_t(p[2]) << 16 | uint32_t(p[3]) << 24;
}

}  // namespace

extern "C" {

// ------------------------------------------------------------------ tokens
RT_API int rt_tokens_open(const char* path, rt_tokens** out) {
  if (!path || !out) return RT_ERR_ARG;
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return RT_ERR_ARG;
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 4) {
    close(fd);
    return RT_ERR_SHAPE;
  }
  void* p = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return RT_ERR_ARG;
  rt_tokens* t = new rt_tokens();
  t->data = static_cast<const uint16_t*>(p);
  t->bytes = static_cast<size_t>(st.st_size);
  t->n = static_cast<int64_t>(st.st_size / 2);
  *out = t;
  return RT_OK;
}

RT_API int rt_tokens_close(rt_tokens* t) {
  if (!t) return RT_ERR_ARG;
  munmap(const_cast<uint16_t*>(t->data), t->bytes);
  delete t;
  return RT_OK;
}

RT_API int rt_tokens_len(const rt_tokens* t, int64_t* n_out) {
  if (!t || !n_out) return RT_ERR_ARG;
  *n_out = t->n;
  return RT_OK;
}

// tokens [start, start + len) as u32 (little-endian u16 on disk).
RT_API int rt_tokens_read(const rt_tokens* t, int64_t start, int64_t len, uint32_t* out) {
  if (!t || !out || start < 0 || len < 0 || start + len > t->n) return RT_ERR_ARG;
  const unsigned char* b = reinterpret_cast<const unsigned char*>(t->data) + 2 * start;
  for (int64_t i = 0; i < len; ++i) out[i] = uint32_t(b[2 * i]) | uint32_t(b[2 * i + 1]) << 8;
  return RT_OK;
}

// The training window of microbatch `micro` at `step`: pos = (step * 7919 +
// micro * 104729) mod (n - seq - 1) (bin/train.rs:285-286, data.rs:92-95);
// tokens = data[pos, pos + seq), targets = data[pos + 1, pos + seq + 1).
RT_API int rt_tokens_train_window(const rt_tokens* t, uint32_t step, uint32_t micro, int seq, uint32_t* tokens,
                                  uint32_t* targets) {
  if (!t || !tokens || !targets || seq <= 0 || t->n < int64_t(seq) + 2) return RT_ERR_ARG;
  const uint64_t max_pos = static_cast<uint64_t>(t->n - seq - 1);
  const uint64_t pos = (uint64_t(step) * 7919u + uint64_t(micro) * 104729u) % max_pos;
  int rc = rt_tokens_read(t, static_cast<int64_t>(pos), seq, tokens);
  return rc ? rc : rt_tokens_read(t, static_cast<int64_t>(pos) + 1, seq, targets);
}

// The validation window `vs`: pos = (vs * seq) mod (n - seq - 1) (bin/train.rs:128-131).
RT_API int rt_tokens_val_window(const rt_tokens* t, uint32_t vs, int seq, uint32_t* tokens, uint32_t* targets) {
  if (!t || !tokens || !targets || seq <= 0 || t->n < int64_t(seq) + 2) return RT_ERR_ARG;
  const uint64_t max_pos = static_cast<uint64_t>(t->n - seq - 1);
  const uint64_t pos = (uint64_t(vs) * uint64_t(seq)) % max_pos;
  int rc = rt_tokens_read(t, static_cast<int64_t>(pos), seq, tokens);
  return rc ? rc : rt_tokens_read(t, static_cast<int64_t>(pos) + 1, seq, targets);
}

// compute_bpb (data.rs:67-89): tokens whose byte length is > 0 count; nats are
// summed in f32 in order; bpb = nats / (ln 2 * bytes), 0 when no byte counts.
RT_API int rt_compute_bpb(const float* losses, const uint32_t* targets, int64_t n, const int32_t* token_bytes,
                          int32_t n_token_bytes, float* bpb_out, float* nats_out, int64_t* bytes_out) {
  if (!losses || !targets || !token_bytes || n < 0) return RT_ERR_ARG;
  float nats = 0.f;
  int64_t bytes = 0;
  for (int64_t i = 0; i < n; ++i) {
    if (targets[i] >= static_cast<uint32_t>(n_token_bytes)) return RT_ERR_TOKEN;
    const int32_t bl = token_bytes[targets[i]];
    if (bl > 0) {
      nats += losses[i];
      bytes += bl;
    }
  }
  if (bpb_out) *bpb_out = bytes > 0 ? nats / (0.69314718f * static_cast<float>(bytes)) : 0.f;
  if (nats_out) *nats_out = nats;
  if (bytes_out) *bytes_out = bytes;
  return RT_OK;
}

// -------------------------------------------------------------- checkpoint
// RSTK (bin/train.rs:165-202): "RSTK", u32 version, u32 step, u32 dim, nlayers,
// vocab, seq (little-endian), then fp32 embed, gamma_final and per layer
// wq wk wv wo w1 w3 w2 gamma1 gamma2.  Version 1 is the reference's file
// byte for byte; version 2 (m and v given) appends the AdamW moments m then v
// in the same order, which the reference does not save.
RT_API int rt_checkpoint_write(const char* path, const rt_model_config* cfg, uint32_t step, const rt_model_ptrs* w,
                               const rt_model_ptrs* m, const rt_model_ptrs* v) {
  if (!path || !cfg || !w || (!m) != (!v)) return RT_ERR_ARG;
  FILE* f = fopen(path, "wb");
  if (!f) return RT_ERR_ARG;
  unsigned char h[28];
  memcpy(h, "RSTK", 4);
  put_u32(h + 4, m ? 2u : 1u);
  put_u32(h + 8, step);
  put_u32(h + 12, static_cast<uint32_t>(cfg->dim));
  put_u32(h + 16, static_cast<uint32_t>(cfg->nlayers));
  put_u32(h + 20, static_cast<uint32_t>(cfg->vocab));
  put_u32(h + 24, static_cast<uint32_t>(cfg->seq));
  bool ok = fwrite(h, 1, sizeof(h), f) == sizeof(h) && write_model(f, *cfg, *w);
  if (ok && m) ok = write_model(f, *cfg, *m) && write_model(f, *cfg, *v);
  ok = (fclose(f) == 0) && ok;
  return ok ? RT_OK : RT_ERR_ARG;
}

// Reads a version 1 or 2 file written for `cfg` (header fields must match);
// m and v are filled when the file has them and they are given.  version_out
// and step_out are optional.
RT_API int rt_checkpoint_read(const char* path, const rt_model_config* cfg, uint32_t* step_out, uint32_t* version_out,
                              const rt_model_ptrs* w, const rt_model_ptrs* m, const rt_model_ptrs* v) {
  if (!path || !cfg || !w || (!m) != (!v)) return RT_ERR_ARG;
  FILE* f = fopen(path, "rb");
  if (!f) return RT_ERR_ARG;
  unsigned char h[28];
  int rc = RT_OK;
  uint32_t version = 0;
  if (fread(h, 1, sizeof(h), f) != sizeof(h) || memcmp(h, "RSTK", 4) != 0) rc = RT_ERR_SHAPE;
  if (rc == RT_OK) {
    version = get_u32(h + 4);
    if ((version != 1 && version != 2) || get_u32(h + 12) != uint32_t(cfg->dim) ||
        get_u32(h + 16) != uint32_t(cfg->nlayers) || get_u32(h + 20) != uint32_t(cfg->vocab) ||
        get_u32(h + 24) != uint32_t(cfg->seq))
      rc = RT_ERR_SHAPE;
  }
  if (rc == RT_OK && !read_model(f, *cfg, *w)) rc = RT_ERR_SHAPE;
  if (rc == RT_OK && version == 2 && m && !(read_model(f, *cfg, *m) && read_model(f, *cfg, *v))) rc = RT_ERR_SHAPE;
  fclose(f);
  if (rc == RT_OK) {
    if (step_out) *step_out = get_u32(h + 8);
    if (version_out) *version_out = version;
  }
  return rc;
}

}  // extern "C"
