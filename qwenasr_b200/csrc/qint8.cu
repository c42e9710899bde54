// qint8.cu -- the .qint8 model file (crates/qwen-asr/src/quantize.rs:1-35,
// 130-346) and the V2 load path of QwenCtx::load (context.rs:341-420):
//
//   * qasr_qint8_open: QuantFile::open -- mmap the file read-only, check the
//     V1 / V2 magic, parse the tensor table (V1 infers the dtype from the
//     scale offset: 0 = F32, else INT8; V2 has an explicit dtype byte); data
//     offsets are relative to the first byte after the table;
//   * qasr_qint8_detect: the model configuration from the tensor shapes
//     (QwenConfig::detect, config.rs:110-156);
//   * qasr_qint8_load_decoder / _load_encoder: DecoderInt8::load
//     (decoder.rs:680-748) and EncoderInt8::load_from_qint8
//     (encoder.rs:466-520) into the device engines.  INT8 matrices and their
//     scales go from the mapping straight to the device; the gate/up
//     interleave of the fused MLP matrix runs on the device
//     (qasr_decoder_set_gate_up); vectors stored as BF16 or INT8 are widened
//     to f32 on the host as QuantFile::get_f32 does.
//
// Host code only; opening and parsing need no GPU.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"

namespace {

const unsigned char kMagicV1[8] = {'Q', 'I', 'N', 'T', '8', 1, 0, 0};
const unsigned char kMagicV2[8] = {'Q', 'I', 'N', 'T', '8', 2, 0, 0};
constexpr int kMaxDims = 8;

struct Tensor {
  std::string name;
  int dtype = 0;  // 0 INT8, 1 F32, 2 BF16
  int n_dims = 0;
  int64_t shape[kMaxDims] = {};
  uint64_t data_off = 0, scale_off = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (int i = 0; i < n_dims; ++i) n *= shape[i];
    return n_dims ? n : 0;
  }
  int64_t bytes() const { return numel() * (dtype == 0 ? 1 : dtype == 1 ? 4 : 2); }
};

uint16_t rd16(const unsigned char *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
uint32_t rd32(const unsigned char *p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
uint64_t rd64(const unsigned char *p) { return (uint64_t)rd32(p) | ((uint64_t)rd32(p + 4) << 32); }

}  // namespace

struct qasr_qint8 {
  unsigned char *map = nullptr;
  size_t size = 0;
  size_t data_start = 0;  // first byte after the tensor table
  int version = 0;
  std::vector<Tensor> tensors;
  std::unordered_map<std::string, int> index;
  const unsigned char *data(const Tensor &t) const { return map + data_start + t.data_off; }
  const float *scales(const Tensor &t) const {
    return t.dtype == 0 ? reinterpret_cast<const float *>(map + data_start + t.scale_off) : nullptr;
  }
  const Tensor *find(const std::string &name) const {
    auto it = index.find(name);
    return it == index.end() ? nullptr : &tensors[it->second];
  }
};

using qasr::set_error;

extern "C" void qasr_qint8_close(qasr_qint8 *f) {
  if (!f) return;
  if (f->map) munmap(f->map, f->size);
  delete f;
}

// QuantFile::open (quantize.rs:130-280), with every table entry and every
// tensor's bytes checked against the file size (the reference stops parsing
// at a truncated entry; here a truncated or out-of-range file is an error).
extern "C" qasr_qint8 *qasr_qint8_open(const char *path) {
  if (!path) {
    set_error("qasr_qint8_open: NULL path");
    return nullptr;
  }
  const int fd = open(path, O_RDONLY);
  if (fd < 0) {
    set_error("qasr_qint8_open: cannot open %s", path);
    return nullptr;
  }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 16) {
    close(fd);
    set_error("qasr_qint8_open: %s is not a .qint8 file (size)", path);
    return nullptr;
  }
  const size_t size = (size_t)st.st_size;
  void *m = mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) {
    set_error("qasr_qint8_open: mmap of %s failed", path);
    return nullptr;
  }
  qasr_qint8 *f = new qasr_qint8();
  f->map = static_cast<unsigned char *>(m);
  f->size = size;
  auto fail = [&](const char *why) -> qasr_qint8 * {
    set_error("qasr_qint8_open: %s: %s", path, why);
    qasr_qint8_close(f);
    return nullptr;
  };
  if (!std::memcmp(f->map, kMagicV2, 8))
    f->version = 2;
  else if (!std::memcmp(f->map, kMagicV1, 8))
    f->version = 1;
  else
    return fail("bad magic");
  const uint32_t n = rd32(f->map + 8);
  size_t pos = 16;
  f->tensors.reserve(n);
  for (uint32_t i = 0; i < n; ++i) {
    Tensor t;
    if (pos + 2 > size) return fail("truncated tensor table");
    const size_t name_len = rd16(f->map + pos);
    pos += 2;
    if (pos + name_len > size) return fail("truncated tensor name");
    t.name.assign(reinterpret_cast<const char *>(f->map + pos), name_len);
    pos += name_len;
    if (f->version == 2) {
      if (pos + 1 > size) return fail("truncated dtype");
      const int d = f->map[pos++];
      t.dtype = (d == 1 || d == 2) ? d : 0;  // unknown tags read as INT8 (quantize.rs:206-211)
    }
    if (pos + 1 > size) return fail("truncated dims");
    t.n_dims = f->map[pos++];
    if (t.n_dims > kMaxDims) return fail("more than 8 dimensions");
    if (pos + 4 * (size_t)t.n_dims + 16 > size) return fail("truncated shape / offsets");
    for (int d = 0; d < t.n_dims; ++d, pos += 4) t.shape[d] = rd32(f->map + pos);
    t.data_off = rd64(f->map + pos);
    t.scale_off = rd64(f->map + pos + 8);
    pos += 16;
    if (f->version == 1) t.dtype = t.scale_off == 0 ? 1 : 0;  // quantize.rs:236-241
    f->index[t.name] = (int)f->tensors.size();
    f->tensors.push_back(std::move(t));
  }
  f->data_start = pos;
  for (const Tensor &t : f->tensors) {
    const size_t avail = size - f->data_start;
    if (t.data_off > avail || (uint64_t)t.bytes() > avail - t.data_off) return fail("tensor data past the end");
    if (t.dtype == 0 && t.n_dims > 0 &&
        (t.scale_off > avail || (uint64_t)t.shape[0] * 4 > avail - t.scale_off))
      return fail("tensor scales past the end");
  }
  return f;
}

extern "C" int qasr_qint8_version(const qasr_qint8 *f) { return f ? f->version : 0; }
extern "C" int qasr_qint8_count(const qasr_qint8 *f) { return f ? (int)f->tensors.size() : 0; }

extern "C" int qasr_qint8_find(const qasr_qint8 *f, const char *name) {
  if (!f || !name) return -1;
  auto it = f->index.find(name);
  return it == f->index.end() ? -1 : it->second;
}

extern "C" int qasr_qint8_tensor(const qasr_qint8 *f, int i, const char **name, int *dtype, int *n_dims,
                                 int64_t *shape, const void **data, const float **scales) {
  if (!f || i < 0 || i >= (int)f->tensors.size()) {
    set_error("qasr_qint8_tensor: no tensor %d", i);
    return QASR_ERR_INVALID;
  }
  const Tensor &t = f->tensors[i];
  if (name) *name = t.name.c_str();
  if (dtype) *dtype = t.dtype;
  if (n_dims) *n_dims = t.n_dims;
  if (shape)
    for (int d = 0; d < t.n_dims; ++d) shape[d] = t.shape[d];
  if (data) *data = f->data(t);
  if (scales) *scales = f->scales(t);
  return QASR_OK;
}

namespace {

const char *kDec = "thinker.model.", *kEnc = "thinker.audio_tower.";

std::string nm(const char *prefix, const std::string &rest) { return std::string(prefix) + rest; }
std::string layer_nm(const char *prefix, int i, const char *rest) {
  return std::string(prefix) + "layers." + std::to_string(i) + "." + rest;
}

int count_layers(const qasr_qint8 *f, const char *prefix) {
  int n = 0;
  while (f->find(layer_nm(prefix, n, "self_attn.q_proj.weight"))) ++n;
  return n;
}

// QuantFile::get_f32 (quantize.rs:292-330) for a tensor of n values: a
// pointer into the mapping for F32, otherwise a widened copy in `buf`.
int vec_f32(const qasr_qint8 *f, const std::string &name, int64_t n, std::vector<float> &buf, const float **out) {
  const Tensor *t = f->find(name);
  if (!t) {
    set_error("qint8: tensor %s missing", name.c_str());
    return QASR_ERR_INVALID;
  }
  if (t->numel() != n) {
    set_error("qint8: %s has %lld values, %lld expected", name.c_str(), (long long)t->numel(), (long long)n);
    return QASR_ERR_INVALID;
  }
  const unsigned char *p = f->data(*t);
  if (t->dtype == 1) {
    *out = reinterpret_cast<const float *>(p);  // copied byte-wise to the device: alignment does not matter
    return QASR_OK;
  }
  buf.resize((size_t)n);
  if (t->dtype == 2) {  // bf16: the high half of an f32
    for (int64_t i = 0; i < n; ++i) {
      const uint32_t u = (uint32_t)rd16(p + 2 * i) << 16;
      std::memcpy(&buf[i], &u, 4);
    }
  } else {  // INT8 [out, in] with row scales: f32(q) * scale
    if (t->n_dims < 2) {
      set_error("qint8: INT8 tensor %s has no rows", name.c_str());
      return QASR_ERR_INVALID;
    }
    const int64_t rows = t->shape[0], cols = n / rows;
    const unsigned char *sp = f->map + f->data_start + t->scale_off;
    for (int64_t r = 0; r < rows; ++r) {
      float s;
      std::memcpy(&s, sp + 4 * r, 4);
      for (int64_t c = 0; c < cols; ++c) buf[r * cols + c] = (float)(int8_t)p[r * cols + c] * s;
    }
  }
  *out = buf.data();
  return QASR_OK;
}

// An INT8 matrix [rows, cols] (QuantFile::get_quant_weight, quantize.rs:274-290).
int mat_i8(const qasr_qint8 *f, const std::string &name, int64_t rows, int64_t cols, const int8_t **q,
           const float **s) {
  const Tensor *t = f->find(name);
  if (!t) {
    set_error("qint8: tensor %s missing", name.c_str());
    return QASR_ERR_INVALID;
  }
  if (t->dtype != 0 || t->n_dims != 2 || t->shape[0] != rows || t->shape[1] != cols) {
    set_error("qint8: %s is not an INT8 [%lld, %lld] matrix", name.c_str(), (long long)rows, (long long)cols);
    return QASR_ERR_INVALID;
  }
  *q = reinterpret_cast<const int8_t *>(f->data(*t));
  *s = f->scales(*t);
  return QASR_OK;
}

bool is_i8(const qasr_qint8 *f, const std::string &name) {
  const Tensor *t = f->find(name);
  return t && t->dtype == 0;
}

}  // namespace

// QwenConfig::detect (config.rs:110-156), every field read from the tensor
// shapes (which gives the reference's values on both published checkpoints):
// decoder hidden and vocabulary from the embedding table, intermediate from
// layer 0's gate projection, layer counts by probing, heads from the q/k
// projections over the head size (the q-norm length), encoder width / FFN /
// output from its q, fc1 and proj2 matrices (64-wide heads, 100-frame chunks,
// 800-frame attention windows).  max_batch / max_seq are left as passed in.
extern "C" int qasr_qint8_detect(const qasr_qint8 *f, qasr_decoder_config *dec, qasr_encoder_config *enc) {
  if (!f) {
    set_error("qasr_qint8_detect: NULL file");
    return QASR_ERR_INVALID;
  }
  if (dec) {
    const Tensor *emb = f->find(nm(kDec, "embed_tokens.weight"));
    const Tensor *gate = f->find(layer_nm(kDec, 0, "mlp.gate_proj.weight"));
    const Tensor *qp = f->find(layer_nm(kDec, 0, "self_attn.q_proj.weight"));
    const Tensor *kp = f->find(layer_nm(kDec, 0, "self_attn.k_proj.weight"));
    const Tensor *qn = f->find(layer_nm(kDec, 0, "self_attn.q_norm.weight"));
    if (!emb || emb->n_dims != 2 || !gate || !qp || !kp) {
      set_error("qasr_qint8_detect: decoder tensors missing (needs a V2 file with the embedding table)");
      return QASR_ERR_INVALID;
    }
    dec->vocab = (int)emb->shape[0];
    dec->hidden = (int)emb->shape[1];
    dec->inter = (int)gate->shape[0];
    dec->n_layers = count_layers(f, kDec);
    dec->head_dim = qn ? (int)qn->numel() : 128;
    dec->n_heads = (int)(qp->shape[0] / dec->head_dim);
    dec->n_kv_heads = (int)(kp->shape[0] / dec->head_dim);
    dec->eps = 1e-6f;
    dec->theta = 1e6f;
    dec->embed_is_int8 = emb->dtype == 0 ? 1 : 0;
  }
  if (enc) {
    const Tensor *qp = f->find(layer_nm(kEnc, 0, "self_attn.q_proj.weight"));
    const Tensor *fc1 = f->find(layer_nm(kEnc, 0, "fc1.weight"));
    const Tensor *p2 = f->find(nm(kEnc, "proj2.weight"));
    if (!qp || !fc1 || !p2) {
      set_error("qasr_qint8_detect: encoder tensors missing (a V1 file keeps the encoder in safetensors)");
      return QASR_ERR_INVALID;
    }
    enc->d_model = (int)qp->shape[0];
    enc->head_dim = 64;
    enc->n_heads = enc->d_model / 64;
    enc->n_layers = count_layers(f, kEnc);
    enc->ffn_dim = (int)fc1->shape[0];
    enc->output_dim = (int)p2->shape[0];
    enc->chunk_size = 100;
    enc->n_window_infer = 800;
  }
  return QASR_OK;
}

// DecoderInt8::load (decoder.rs:680-748) into an engine created with the
// detected configuration: per layer the q/k/v/o/down INT8 matrices and norms
// (qasr_decoder_set_layer), gate and up interleaved on the device
// (qasr_decoder_set_gate_up); then the embedding table, final norm and the
// lm head (tied to the INT8 embedding table when the file has none).
extern "C" int qasr_qint8_load_decoder(const qasr_qint8 *f, qasr_decoder *dec) {
  const qasr_decoder_config *c = qasr_decoder_get_config(dec);
  if (!f || !c) {
    set_error("qasr_qint8_load_decoder: NULL argument");
    return QASR_ERR_INVALID;
  }
  const int64_t H = c->hidden, I = c->inter, hd = c->head_dim, q_dim = (int64_t)c->n_heads * hd,
                kv = (int64_t)c->n_kv_heads * hd;
  if (count_layers(f, kDec) < c->n_layers) {
    set_error("qasr_qint8_load_decoder: the file has %d decoder layers, the engine %d", count_layers(f, kDec),
              c->n_layers);
    return QASR_ERR_INVALID;
  }
  int rc = QASR_OK;
  std::vector<float> b0, b1, b2, b3, bn;
  for (int l = 0; l < c->n_layers && !rc; ++l) {
    qasr_dec_layer_weights w{};
    const int8_t *gate = nullptr, *up = nullptr;
    const float *gate_s = nullptr, *up_s = nullptr;
    auto L = [&](const char *rest) { return layer_nm(kDec, l, rest); };
    if (!rc) rc = mat_i8(f, L("self_attn.q_proj.weight"), q_dim, H, &w.wq, &w.wq_s);
    if (!rc) rc = mat_i8(f, L("self_attn.k_proj.weight"), kv, H, &w.wk, &w.wk_s);
    if (!rc) rc = mat_i8(f, L("self_attn.v_proj.weight"), kv, H, &w.wv, &w.wv_s);
    if (!rc) rc = mat_i8(f, L("self_attn.o_proj.weight"), H, q_dim, &w.wo, &w.wo_s);
    if (!rc) rc = mat_i8(f, L("mlp.gate_proj.weight"), I, H, &gate, &gate_s);
    if (!rc) rc = mat_i8(f, L("mlp.up_proj.weight"), I, H, &up, &up_s);
    if (!rc) rc = mat_i8(f, L("mlp.down_proj.weight"), H, I, &w.down, &w.down_s);
    if (!rc) rc = vec_f32(f, L("self_attn.q_norm.weight"), hd, b0, &w.q_norm);
    if (!rc) rc = vec_f32(f, L("self_attn.k_norm.weight"), hd, b1, &w.k_norm);
    if (!rc) rc = vec_f32(f, L("input_layernorm.weight"), H, b2, &w.input_norm);
    if (!rc) rc = vec_f32(f, L("post_attention_layernorm.weight"), H, b3, &w.post_attn_norm);
    if (!rc) rc = qasr_decoder_set_layer(dec, l, &w);  // gate_up NULL: set below
    if (!rc) rc = qasr_decoder_set_gate_up(dec, l, gate, gate_s, up, up_s);
  }
  if (rc) return rc;
  const Tensor *emb = f->find(nm(kDec, "embed_tokens.weight"));
  if (!emb || emb->n_dims != 2 || emb->shape[0] != c->vocab || emb->shape[1] != H) {
    set_error("qasr_qint8_load_decoder: embedding table missing or not [%d, %lld]", c->vocab, (long long)H);
    return QASR_ERR_INVALID;
  }
  if ((emb->dtype == 0) != (c->embed_is_int8 != 0)) {
    set_error("qasr_qint8_load_decoder: embed_is_int8 = %d but the file's table has dtype %d", c->embed_is_int8,
              emb->dtype);
    return QASR_ERR_INVALID;
  }
  const void *table = nullptr;
  const float *table_s = nullptr;
  std::vector<float> wide;
  if (emb->dtype == 0) {
    table = f->data(*emb);
    table_s = f->scales(*emb);
  } else {
    const float *p = nullptr;
    if ((rc = vec_f32(f, nm(kDec, "embed_tokens.weight"), (int64_t)c->vocab * H, wide, &p))) return rc;
    table = p;
  }
  const float *norm = nullptr;
  if ((rc = vec_f32(f, nm(kDec, "norm.weight"), H, bn, &norm))) return rc;
  const int8_t *lm = nullptr;
  const float *lm_s = nullptr;
  if (f->find("thinker.lm_head.weight") &&
      (rc = mat_i8(f, "thinker.lm_head.weight", c->vocab, H, &lm, &lm_s)))
    return rc;
  return qasr_decoder_set_globals(dec, table, table_s, norm, lm, lm_s);
}

// EncoderInt8::load_from_qint8 (encoder.rs:466-520): f32 convolutions, INT8
// projections (each group falls back to widened f32 weights when the file
// stores it as F32 / BF16), f32 biases and norms.
extern "C" int qasr_qint8_load_encoder(const qasr_qint8 *f, qasr_encoder *enc) {
  const qasr_encoder_config *c = qasr_encoder_get_config(enc);
  if (!f || !c) {
    set_error("qasr_qint8_load_encoder: NULL argument");
    return QASR_ERR_INVALID;
  }
  if (count_layers(f, kEnc) < c->n_layers) {
    set_error("qasr_qint8_load_encoder: the file has %d encoder layers, the engine %d", count_layers(f, kEnc),
              c->n_layers);
    return QASR_ERR_INVALID;
  }
  const int64_t D = c->d_model, F = c->ffn_dim, O = c->output_dim, CH = 480, h3 = 16;
  int rc = QASR_OK;
  // conv stem (f32) and conv_out
  std::vector<float> cb[7];
  const float *cw[7] = {};
  const char *conv_names[6] = {"conv2d1.weight", "conv2d1.bias", "conv2d2.weight",
                               "conv2d2.bias",   "conv2d3.weight", "conv2d3.bias"};
  const int64_t conv_n[6] = {CH * 9, CH, CH * CH * 9, CH, CH * CH * 9, CH};
  for (int i = 0; i < 6 && !rc; ++i) rc = vec_f32(f, nm(kEnc, conv_names[i]), conv_n[i], cb[i], &cw[i]);
  if (rc) return rc;
  const std::string co = nm(kEnc, "conv_out.weight");
  if (is_i8(f, co)) {
    const int8_t *q = nullptr;
    const float *s = nullptr;
    if ((rc = mat_i8(f, co, D, CH * h3, &q, &s))) return rc;
    rc = qasr_encoder_set_conv_int8(enc, cw[0], cw[1], cw[2], cw[3], cw[4], cw[5], q, s);
  } else {
    if ((rc = vec_f32(f, co, D * CH * h3, cb[6], &cw[6]))) return rc;
    rc = qasr_encoder_set_conv(enc, cw[0], cw[1], cw[2], cw[3], cw[4], cw[5], cw[6]);
  }
  if (rc) return rc;
  const char *mats[6] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                         "self_attn.out_proj.weight", "fc1.weight", "fc2.weight"};
  const int64_t mrows[6] = {D, D, D, D, F, D}, mcols[6] = {D, D, D, D, D, F};
  const char *vecs[10] = {"self_attn_layer_norm.weight", "self_attn_layer_norm.bias", "self_attn.q_proj.bias",
                          "self_attn.k_proj.bias",       "self_attn.v_proj.bias",     "self_attn.out_proj.bias",
                          "final_layer_norm.weight",     "final_layer_norm.bias",     "fc1.bias",
                          "fc2.bias"};
  const int64_t vlen[10] = {D, D, D, D, D, D, D, D, F, D};
  std::vector<float> vb[10], mb[6];
  for (int l = 0; l < c->n_layers && !rc; ++l) {
    const float *v[10] = {};
    for (int i = 0; i < 10 && !rc; ++i) rc = vec_f32(f, layer_nm(kEnc, l, vecs[i]), vlen[i], vb[i], &v[i]);
    if (rc) break;
    bool all_i8 = true;
    for (int i = 0; i < 6; ++i) all_i8 = all_i8 && is_i8(f, layer_nm(kEnc, l, mats[i]));
    if (all_i8) {
      const int8_t *q[6] = {};
      const float *s[6] = {};
      for (int i = 0; i < 6 && !rc; ++i) rc = mat_i8(f, layer_nm(kEnc, l, mats[i]), mrows[i], mcols[i], &q[i], &s[i]);
      if (rc) break;
      qasr_enc_layer_weights_int8 w{v[0], v[1], q[0], s[0], v[2], q[1], s[1], v[3], q[2], s[2], v[4],
                                    q[3], s[3], v[5], v[6], v[7], q[4], s[4], v[8], q[5], s[5], v[9]};
      rc = qasr_encoder_set_layer_int8(enc, l, &w);
    } else {
      const float *m[6] = {};
      for (int i = 0; i < 6 && !rc; ++i)
        rc = vec_f32(f, layer_nm(kEnc, l, mats[i]), mrows[i] * mcols[i], mb[i], &m[i]);
      if (rc) break;
      qasr_enc_layer_weights w{v[0], v[1], m[0], v[2], m[1], v[3], m[2], v[4], m[3], v[5],
                               v[6], v[7], m[4], v[8], m[5], v[9]};
      rc = qasr_encoder_set_layer(enc, l, &w);
    }
  }
  if (rc) return rc;
  // post LayerNorm and projections
  const float *lw = nullptr, *lb = nullptr, *b1 = nullptr, *b2 = nullptr;
  std::vector<float> t0, t1, t2, t3, t4, t5;
  if ((rc = vec_f32(f, nm(kEnc, "ln_post.weight"), D, t0, &lw))) return rc;
  if ((rc = vec_f32(f, nm(kEnc, "ln_post.bias"), D, t1, &lb))) return rc;
  if ((rc = vec_f32(f, nm(kEnc, "proj1.bias"), D, t2, &b1))) return rc;
  if ((rc = vec_f32(f, nm(kEnc, "proj2.bias"), O, t3, &b2))) return rc;
  const std::string p1 = nm(kEnc, "proj1.weight"), p2 = nm(kEnc, "proj2.weight");
  if (is_i8(f, p1) && is_i8(f, p2)) {
    const int8_t *q1 = nullptr, *q2 = nullptr;
    const float *s1 = nullptr, *s2 = nullptr;
    if ((rc = mat_i8(f, p1, D, D, &q1, &s1))) return rc;
    if ((rc = mat_i8(f, p2, O, D, &q2, &s2))) return rc;
    return qasr_encoder_set_post_int8(enc, lw, lb, q1, s1, b1, q2, s2, b2);
  }
  const float *w1 = nullptr, *w2 = nullptr;
  if ((rc = vec_f32(f, p1, D * D, t4, &w1))) return rc;
  if ((rc = vec_f32(f, p2, O * D, t5, &w2))) return rc;
  return qasr_encoder_set_post(enc, lw, lb, w1, b1, w2, b2);
}
