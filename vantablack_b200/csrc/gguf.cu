// gguf.cu -- GGUF v2/v3 files for the CUDA backend: the reader of
// src/core/parser.zig (header, typed metadata, tensor descriptors) and
// src/core/mapper.zig (read-only mmap, bounds-checked tensor slices), and the
// llama mapping of src/runtime/model.zig (LlamaConfig.fromCatalog, Model.init)
// feeding vtb_cuda_model_create.  Host code only; all numbers little-endian.
//
// Same accept/reject rules as the reference parser: magic 'GGUF', version 2
// or 3, metadata value types 0..12, arrays nested at most 4 deep, tensor
// element counts that overflow u64 or do not fill whole quantization blocks
// are refused, general.alignment (u32) defaults to 32, and a tensor's bytes
// must lie inside the file.  One addition: an alignment that is not a power
// of two is refused (the reference's align-up assumes one).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/vtb_cuda.h"
#include "common.cuh"

namespace {

enum MetaType : uint32_t {
  M_U8 = 0, M_I8 = 1, M_U16 = 2, M_I16 = 3, M_U32 = 4, M_I32 = 5, M_F32 = 6, M_BOOL = 7,
  M_STRING = 8, M_ARRAY = 9, M_U64 = 10, M_I64 = 11, M_F64 = 12,
};
constexpr uint32_t kMaxArrayDepth = 4;

struct Meta {
  std::string key;
  uint32_t type = 0;
  bool is_signed = false, is_float = false;
  uint64_t u = 0;  // unsigned / bool values
  int64_t i = 0;   // signed values
  double f = 0;    // float values
  uint64_t off = 0, len = 0;  // string bytes, or an array's payload, inside the map
  uint32_t arr_type = 0;
  uint64_t arr_count = 0;
};

struct Tensor {
  std::string name;
  std::vector<uint64_t> dims;
  uint32_t type = 0;
  uint64_t rel = 0, size = 0;
};

// Bytes per block and elements per block of the ggml types (ggml-quants.h;
// parser.zig blockInfo).  0 = size unknown (the tensor is still listed).
void block_info(uint32_t t, uint64_t* el, uint64_t* by) {
  struct E { uint32_t t; uint64_t el, by; };
  static const E tab[] = {{0, 1, 4},    {1, 1, 2},    {30, 1, 2},   {28, 1, 8},    {24, 1, 1},   {25, 1, 2},
                          {26, 1, 4},   {27, 1, 8},   {8, 32, 34},  {2, 32, 18},   {3, 32, 20},  {6, 32, 22},
                          {7, 32, 24},  {9, 32, 36},  {10, 256, 84}, {11, 256, 110}, {12, 256, 144}, {13, 256, 176},
                          {14, 256, 210}, {15, 256, 292}, {31, 256, 54}, {32, 256, 66}};
  for (const E& e : tab)
    if (e.t == t) {
      *el = e.el;
      *by = e.by;
      return;
    }
  *el = 0;
  *by = 0;
}

struct Cursor {
  const uint8_t* p;
  size_t n, off = 0;
  const char* err = nullptr;  // first failure
  bool need(size_t k) {
    if (err) return false;
    if (k > n - off) {
      err = "unexpected end of file";
      return false;
    }
    return true;
  }
  template <typename T>
  T get() {
    T v{};
    if (need(sizeof(T))) {
      memcpy(&v, p + off, sizeof(T));  // little-endian host; unaligned-safe
      off += sizeof(T);
    }
    return v;
  }
  bool str(uint64_t* o, uint64_t* l) {
    const uint64_t len = get<uint64_t>();
    if (err || !need(len)) return false;
    *o = off;
    *l = len;
    off += len;
    return true;
  }
};

bool read_value(Cursor& c, uint32_t t, uint32_t depth, Meta* m) {
  if (depth > kMaxArrayDepth) {
    c.err = "array nesting too deep";
    return false;
  }
  switch (t) {
    case M_U8: m->u = c.get<uint8_t>(); break;
    case M_I8: m->i = c.get<int8_t>(); m->is_signed = true; break;
    case M_U16: m->u = c.get<uint16_t>(); break;
    case M_I16: m->i = c.get<int16_t>(); m->is_signed = true; break;
    case M_U32: m->u = c.get<uint32_t>(); break;
    case M_I32: m->i = c.get<int32_t>(); m->is_signed = true; break;
    case M_U64: m->u = c.get<uint64_t>(); break;
    case M_I64: m->i = c.get<int64_t>(); m->is_signed = true; break;
    case M_F32: m->f = c.get<float>(); m->is_float = true; break;
    case M_F64: m->f = c.get<double>(); m->is_float = true; break;
    case M_BOOL: m->u = c.get<uint8_t>() != 0; break;
    case M_STRING: c.str(&m->off, &m->len); break;
    case M_ARRAY: {
      const uint32_t et = c.get<uint32_t>();
      const uint64_t count = c.get<uint64_t>();
      if (c.err) return false;
      if (et > M_F64) {
        c.err = "unknown metadata value type";
        return false;
      }
      const size_t start = c.off;
      Meta scratch;
      for (uint64_t k = 0; k < count && !c.err; ++k) read_value(c, et, depth + 1, &scratch);  // walk, keep nothing
      m->arr_type = et;
      m->arr_count = count;
      m->off = start;
      m->len = c.off - start;
      break;
    }
    default: c.err = "unknown metadata value type"; return false;
  }
  m->type = t;
  return !c.err;
}

}  // namespace

struct VtbCudaGguf {
  const uint8_t* map = nullptr;
  size_t len = 0;
  uint32_t version = 0, alignment = 32;
  uint64_t data_start = 0;
  std::vector<Meta> meta;
  std::vector<Tensor> tensors;

  const Meta* find_meta(const char* key) const {
    for (const Meta& m : meta)
      if (m.key == key) return &m;
    return nullptr;
  }
  const Tensor* find_tensor(const char* name) const {
    for (const Tensor& t : tensors)
      if (t.name == name) return &t;
    return nullptr;
  }
  // Bounds-checked tensor bytes (mapper.zig tensorSliceFromDesc).
  const uint8_t* slice(const Tensor& t) const {
    const uint64_t start = data_start + t.rel;
    if (start < data_start || start + t.size < start || start + t.size > len) return nullptr;
    return map + start;
  }
};

static int parse(VtbCudaGguf* g) {
  Cursor c{g->map, g->len};
  auto fail = [&](const char* why) { return set_err(VTB_CUDA_ERR_PARSE, "GGUF: %s", why); };
  if (g->len < 24) return fail("file too small for a GGUF header");
  if (c.get<uint32_t>() != 0x46554747u) return fail("not a GGUF file");
  g->version = c.get<uint32_t>();
  if (g->version != 2 && g->version != 3) return fail("unsupported GGUF version");
  const uint64_t n_tensors = c.get<uint64_t>(), n_meta = c.get<uint64_t>();
  // every record takes at least 12 bytes: a count beyond the file is a truncation
  if (n_meta > g->len / 12 || n_tensors > g->len / 12) return fail("unexpected end of file");
  g->meta.resize(n_meta);
  for (uint64_t k = 0; k < n_meta; ++k) {
    Meta& m = g->meta[k];
    uint64_t ko, kl;
    if (!c.str(&ko, &kl)) return fail(c.err);
    m.key.assign(reinterpret_cast<const char*>(g->map + ko), kl);
    const uint32_t t = c.get<uint32_t>();
    if (c.err) return fail(c.err);
    if (!read_value(c, t, 0, &m)) return fail(c.err);
    if (m.key == "general.alignment" && m.type == M_U32) g->alignment = (uint32_t)m.u;
  }
  if (g->alignment == 0 || (g->alignment & (g->alignment - 1))) return fail("alignment is not a power of two");
  g->tensors.resize(n_tensors);
  for (uint64_t k = 0; k < n_tensors; ++k) {
    Tensor& t = g->tensors[k];
    uint64_t no, nl;
    if (!c.str(&no, &nl)) return fail(c.err);
    t.name.assign(reinterpret_cast<const char*>(g->map + no), nl);
    const uint32_t nd = c.get<uint32_t>();
    if (c.err) return fail(c.err);
    if (nd > (g->len - c.off) / 8) return fail("unexpected end of file");
    t.dims.resize(nd);
    uint64_t numel = 1;
    for (uint32_t d = 0; d < nd; ++d) {
      t.dims[d] = c.get<uint64_t>();
      if (t.dims[d] && numel > UINT64_MAX / t.dims[d]) return fail("unsupported tensor block shape");
      numel *= t.dims[d];
    }
    t.type = c.get<uint32_t>();
    t.rel = c.get<uint64_t>();
    if (c.err) return fail(c.err);
    uint64_t el, by;
    block_info(t.type, &el, &by);
    if (el) {
      if (numel % el || numel / el > UINT64_MAX / by) return fail("unsupported tensor block shape");
      t.size = numel / el * by;
    }
  }
  g->data_start = (c.off + g->alignment - 1) & ~(uint64_t)(g->alignment - 1);
  if (g->data_start > g->len) return fail("unexpected end of file");
  return VTB_CUDA_OK;
}

// Unsigned / signed integer metadata as int64 (model.zig metaUsize); negative
// values are refused like the reference's usize cast.
static bool meta_uint(const VtbCudaGguf* g, const std::string& key, int64_t* out) {
  const Meta* m = g->find_meta(key.c_str());
  if (!m || m->is_float || m->type == M_STRING || m->type == M_ARRAY || m->type == M_BOOL) return false;
  if (m->is_signed) {
    if (m->i < 0) return false;
    *out = m->i;
  } else {
    if (m->u > (uint64_t)INT64_MAX) return false;
    *out = (int64_t)m->u;
  }
  return true;
}

static bool meta_float(const VtbCudaGguf* g, const std::string& key, double* out) {
  const Meta* m = g->find_meta(key.c_str());
  if (!m || !m->is_float) return false;
  *out = m->f;
  return true;
}

extern "C" {

VtbCudaGguf* vtb_cuda_gguf_open(const char* path) {
  if (!path) {
    set_err(VTB_CUDA_ERR_INVALID_ARG, "null path");
    return nullptr;
  }
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) {
    set_err(VTB_CUDA_ERR_FILE_OPEN, "GGUF: cannot open %s", path);
    return nullptr;
  }
  struct stat sb;
  if (fstat(fd, &sb) != 0 || sb.st_size <= 0) {
    close(fd);
    set_err(VTB_CUDA_ERR_FILE_OPEN, "GGUF: %s is empty or unreadable", path);
    return nullptr;
  }
  void* p = mmap(nullptr, (size_t)sb.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) {
    set_err(VTB_CUDA_ERR_FILE_OPEN, "GGUF: cannot map %s", path);
    return nullptr;
  }
  VtbCudaGguf* g = new (std::nothrow) VtbCudaGguf();
  if (!g) {
    munmap(p, (size_t)sb.st_size);
    set_err(VTB_CUDA_ERR_OOM, "out of host memory");
    return nullptr;
  }
  g->map = static_cast<const uint8_t*>(p);
  g->len = (size_t)sb.st_size;
  if (parse(g) != VTB_CUDA_OK) {
    vtb_cuda_gguf_close(g);
    return nullptr;
  }
  return g;
}

void vtb_cuda_gguf_close(VtbCudaGguf* g) {
  if (!g) return;
  if (g->map) munmap(const_cast<uint8_t*>(g->map), g->len);
  delete g;
}

int vtb_cuda_gguf_info(const VtbCudaGguf* g, uint32_t* version, uint32_t* alignment, uint64_t* data_offset,
                       int64_t* n_tensors, int64_t* n_meta) {
  if (!g) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null GGUF handle");
  if (version) *version = g->version;
  if (alignment) *alignment = g->alignment;
  if (data_offset) *data_offset = g->data_start;
  if (n_tensors) *n_tensors = (int64_t)g->tensors.size();
  if (n_meta) *n_meta = (int64_t)g->meta.size();
  return VTB_CUDA_OK;
}

int vtb_cuda_gguf_tensor_info(const VtbCudaGguf* g, int64_t i, const char** name, uint32_t* ggml_type,
                              uint32_t* n_dims, uint64_t* dims, uint64_t* rel_offset, uint64_t* size_bytes) {
  if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return set_err(VTB_CUDA_ERR_INVALID_ARG, "bad tensor index");
  const Tensor& t = g->tensors[(size_t)i];
  if (name) *name = t.name.c_str();
  if (ggml_type) *ggml_type = t.type;
  if (n_dims) *n_dims = (uint32_t)t.dims.size();
  if (dims)
    for (size_t d = 0; d < t.dims.size() && d < VTB_CUDA_GGUF_MAX_DIMS; ++d) dims[d] = t.dims[d];
  if (rel_offset) *rel_offset = t.rel;
  if (size_bytes) *size_bytes = t.size;
  return VTB_CUDA_OK;
}

const void* vtb_cuda_gguf_tensor(const VtbCudaGguf* g, const char* name, uint32_t* ggml_type, uint64_t* size_bytes) {
  if (!g || !name) {
    set_err(VTB_CUDA_ERR_INVALID_ARG, "null argument");
    return nullptr;
  }
  const Tensor* t = g->find_tensor(name);
  if (!t) {
    set_err(VTB_CUDA_ERR_INVALID_ARG, "GGUF: tensor %s not found", name);
    return nullptr;
  }
  const uint8_t* p = g->slice(*t);
  if (!p) {
    set_err(VTB_CUDA_ERR_PARSE, "GGUF: tensor %s lies outside the file", name);
    return nullptr;
  }
  if (ggml_type) *ggml_type = t->type;
  if (size_bytes) *size_bytes = t->size;
  return p;
}

int vtb_cuda_gguf_meta_int(const VtbCudaGguf* g, const char* key, int64_t* out) {
  if (!g || !key || !out) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null argument");
  const Meta* m = g->find_meta(key);
  if (!m) return set_err(VTB_CUDA_ERR_INVALID_ARG, "GGUF: no metadata key %s", key);
  if (m->is_float || m->type == M_STRING || m->type == M_ARRAY)
    return set_err(VTB_CUDA_ERR_INVALID_ARG, "GGUF: %s is not an integer", key);
  *out = m->is_signed ? m->i : (int64_t)m->u;
  return VTB_CUDA_OK;
}

int vtb_cuda_gguf_meta_float(const VtbCudaGguf* g, const char* key, double* out) {
  if (!g || !key || !out) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null argument");
  if (!meta_float(g, key, out)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "GGUF: %s is missing or not a float", key);
  return VTB_CUDA_OK;
}

int vtb_cuda_gguf_meta_string(const VtbCudaGguf* g, const char* key, const char** ptr, uint64_t* len) {
  if (!g || !key || !ptr || !len) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null argument");
  const Meta* m = g->find_meta(key);
  if (!m || m->type != M_STRING) return set_err(VTB_CUDA_ERR_INVALID_ARG, "GGUF: %s is missing or not a string", key);
  *ptr = reinterpret_cast<const char*>(g->map + m->off);
  *len = m->len;
  return VTB_CUDA_OK;
}

int vtb_cuda_gguf_meta_array(const VtbCudaGguf* g, const char* key, uint32_t* elem_type, uint64_t* count) {
  if (!g || !key) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null argument");
  const Meta* m = g->find_meta(key);
  if (!m || m->type != M_ARRAY) return set_err(VTB_CUDA_ERR_INVALID_ARG, "GGUF: %s is missing or not an array", key);
  if (elem_type) *elem_type = m->arr_type;
  if (count) *count = m->arr_count;
  return VTB_CUDA_OK;
}

// LlamaConfig.fromCatalog (model.zig:72-146) for the architectures the CUDA
// forward implements (llama).
int vtb_cuda_gguf_llama_config(const VtbCudaGguf* g, VtbCudaLlamaConfig* cfg) {
  if (!g || !cfg) return set_err(VTB_CUDA_ERR_INVALID_ARG, "null argument");
  const Meta* arch = g->find_meta("general.architecture");
  if (!arch || arch->type != M_STRING) return set_err(VTB_CUDA_ERR_PARSE, "GGUF: missing general.architecture");
  const std::string a(reinterpret_cast<const char*>(g->map + arch->off), arch->len);
  if (a != "llama") return set_err(VTB_CUDA_ERR_UNSUPPORTED, "GGUF: architecture %s is not supported", a.c_str());
  int64_t dim, n_layers, n_heads, ffn, ctx, n_kv, vocab;
  if (!meta_uint(g, a + ".embedding_length", &dim) || !meta_uint(g, a + ".block_count", &n_layers) ||
      !meta_uint(g, a + ".attention.head_count", &n_heads) || !meta_uint(g, a + ".feed_forward_length", &ffn) ||
      !meta_uint(g, a + ".context_length", &ctx))
    return set_err(VTB_CUDA_ERR_PARSE, "GGUF: missing llama metadata");
  if (!meta_uint(g, a + ".attention.head_count_kv", &n_kv)) n_kv = n_heads;
  double rope = 10000.0, eps = 1e-5;
  meta_float(g, a + ".rope.freq_base", &rope);
  meta_float(g, a + ".attention.layer_norm_rms_epsilon", &eps);
  if (!meta_uint(g, a + ".vocab_size", &vocab)) {
    const Meta* tok = g->find_meta("tokenizer.ggml.tokens");
    if (!tok || tok->type != M_ARRAY) return set_err(VTB_CUDA_ERR_PARSE, "GGUF: missing vocabulary size");
    vocab = (int64_t)tok->arr_count;
  }
  if (n_heads <= 0) return set_err(VTB_CUDA_ERR_PARSE, "GGUF: zero attention heads");
  const int64_t lim = INT32_MAX;
  if (dim > lim || n_layers > lim || ffn > lim || ctx > lim || n_kv > lim || vocab > lim || n_heads > lim)
    return set_err(VTB_CUDA_ERR_UNSUPPORTED, "GGUF: model dimensions beyond 32 bits");
  cfg->dim = (int32_t)dim;
  cfg->n_layers = (int32_t)n_layers;
  cfg->n_heads = (int32_t)n_heads;
  cfg->n_kv_heads = (int32_t)n_kv;
  cfg->head_dim = (int32_t)(dim / n_heads);
  cfg->ffn_dim = (int32_t)ffn;
  cfg->vocab_size = (int32_t)vocab;
  cfg->max_seq = (int32_t)ctx;
  cfg->rope_base = (float)rope;
  cfg->rms_eps = (float)eps;
  return VTB_CUDA_OK;
}

}  // extern "C"

// Model.init (model.zig:201-243): the llama tensor names, each checked for
// type and [k, rows] shape before the upload.  output.weight falls back to
// token_embd.weight (tied embeddings).
static int gguf_layers(const VtbCudaGguf* g, int32_t max_seq, VtbCudaLlamaConfig* cfg,
                       std::vector<VtbCudaLayerWeights>* layers, const void** embd, int32_t* q_embd,
                       const float** out_norm, const void** out_w, int32_t* q_out) {
  int rc = vtb_cuda_gguf_llama_config(g, cfg);
  if (rc) return rc;
  if (max_seq > 0) cfg->max_seq = max_seq;
  const uint64_t d = (uint64_t)cfg->dim, kvd = (uint64_t)cfg->n_kv_heads * cfg->head_dim, f = (uint64_t)cfg->ffn_dim,
                 v = (uint64_t)cfg->vocab_size, qd = (uint64_t)cfg->n_heads * cfg->head_dim;
  auto fetch = [&](const std::string& name, uint64_t k, uint64_t rows, bool norm, const void** ptr,
                   int32_t* q) -> int {
    const Tensor* t = g->find_tensor(name.c_str());
    if (!t) return set_err(VTB_CUDA_ERR_PARSE, "GGUF: tensor %s not found", name.c_str());
    const bool shape_ok = norm ? (t->dims.size() == 1 && t->dims[0] == k)
                               : (t->dims.size() == 2 && t->dims[0] == k && t->dims[1] == rows);
    if (!shape_ok) return set_err(VTB_CUDA_ERR_PARSE, "GGUF: tensor %s has an unexpected shape", name.c_str());
    if (norm ? t->type != 0 : !host_quant_ok((int)t->type))
      return set_err(VTB_CUDA_ERR_UNSUPPORTED, "GGUF: tensor %s has a ggml type this path does not support",
                     name.c_str());
    const uint8_t* p = g->slice(*t);
    if (!p) return set_err(VTB_CUDA_ERR_PARSE, "GGUF: tensor %s lies outside the file", name.c_str());
    *ptr = p;
    if (q) *q = (int32_t)t->type;
    return VTB_CUDA_OK;
  };
  layers->assign((size_t)cfg->n_layers, VtbCudaLayerWeights{});
  for (int32_t l = 0; l < cfg->n_layers; ++l) {
    VtbCudaLayerWeights& L = (*layers)[(size_t)l];
    const std::string b = "blk." + std::to_string(l) + ".";
    const void* an = nullptr;
    const void* fn = nullptr;
    if ((rc = fetch(b + "attn_norm.weight", d, 0, true, &an, nullptr)) ||
        (rc = fetch(b + "attn_q.weight", d, qd, false, &L.attn_q, &L.q_attn_q)) ||
        (rc = fetch(b + "attn_k.weight", d, kvd, false, &L.attn_k, &L.q_attn_k)) ||
        (rc = fetch(b + "attn_v.weight", d, kvd, false, &L.attn_v, &L.q_attn_v)) ||
        (rc = fetch(b + "attn_output.weight", qd, d, false, &L.attn_o, &L.q_attn_o)) ||
        (rc = fetch(b + "ffn_norm.weight", d, 0, true, &fn, nullptr)) ||
        (rc = fetch(b + "ffn_gate.weight", d, f, false, &L.ffn_gate, &L.q_ffn_gate)) ||
        (rc = fetch(b + "ffn_up.weight", d, f, false, &L.ffn_up, &L.q_ffn_up)) ||
        (rc = fetch(b + "ffn_down.weight", f, d, false, &L.ffn_down, &L.q_ffn_down)))
      return rc;
    L.attn_norm = static_cast<const float*>(an);
    L.ffn_norm = static_cast<const float*>(fn);
  }
  const void* on = nullptr;
  if ((rc = fetch("token_embd.weight", d, v, false, embd, q_embd)) ||
      (rc = fetch("output_norm.weight", d, 0, true, &on, nullptr)))
    return rc;
  *out_norm = static_cast<const float*>(on);
  if (g->find_tensor("output.weight")) {
    rc = fetch("output.weight", d, v, false, out_w, q_out);
    if (rc) return rc;
  } else {
    *out_w = *embd;
    *q_out = *q_embd;
  }
  return VTB_CUDA_OK;
}

extern "C" {

VtbCudaModel* vtb_cuda_model_create_gguf_tp(VtbCudaCtx* ctx, VtbCudaTp* tp, const VtbCudaGguf* g, int32_t max_seq) {
  if (!g) {
    set_err(VTB_CUDA_ERR_INVALID_ARG, "null GGUF handle");
    return nullptr;
  }
  VtbCudaLlamaConfig cfg;
  std::vector<VtbCudaLayerWeights> layers;
  const void *embd = nullptr, *out_w = nullptr;
  const float* out_norm = nullptr;
  int32_t q_embd = 0, q_out = 0;
  if (gguf_layers(g, max_seq, &cfg, &layers, &embd, &q_embd, &out_norm, &out_w, &q_out)) return nullptr;
  return vtb_cuda_model_create_tp(ctx, tp, &cfg, layers.data(), embd, q_embd, out_norm, out_w, q_out);
}

VtbCudaModel* vtb_cuda_model_create_gguf(VtbCudaCtx* ctx, const VtbCudaGguf* g, int32_t max_seq) {
  return vtb_cuda_model_create_gguf_tp(ctx, nullptr, g, max_seq);
}

}  // extern "C"
