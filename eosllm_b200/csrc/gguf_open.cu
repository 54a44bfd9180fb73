// gguf_open.cu -- GGUF v3 Llama-family models straight to the device
// decoder.  The reference engine reads the whole file into host memory
// (src/format/gguf/gguf.c:445-453) and the text modality looks its tensors
// up by name (src/modality/text/text.c:104-215).  Here the file is mapped
// read-only, parsed with the same rules, and the decoder description's
// tensor pointers point into the mapping; eosi_cuda_text_open then copies
// only this rank's rows / columns of every matrix to its GPU, so a
// tensor-parallel rank reads (pages in) only its own shard of the file.
//
// Container rules mirrored from gguf.c: magic "GGUF", version 3 only
// (:462-467); metadata value types 0..12 with arrays of scalars or strings
// (:130-140, :228-290); tensor rank 1..6, every dimension 1..2^32-1, element
// counts without u64 overflow (:605-627); tensor types F32 / F16 / Q8_0 / Q4_K
// (:148-156) whose element count divides into whole blocks (:158-175);
// general.alignment a power of two (default 32, :579-590); tensor data
// inside the file after the aligned data offset (:652-680).
// Model rules mirrored from eosi_text_open (text.c:104-160): keys in the
// `<general.architecture>.` namespace; embedding_length, block_count,
// attention.head_count, feed_forward_length and context_length required
// (unsigned or signed integer or bool values); head_count_kv defaults to
// head_count; rope.freq_base (F32) defaults to 10000, layer_norm_rms_epsilon
// (F32) to 1e-5; max_ctx = min(context_length, the caller's bound when
// non-zero); n_vocab = token_embd's second dimension; output.weight absent
// means tied to the embedding (which this decoder does not support: F16).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <unordered_map>
#include <vector>

#include "eos_common.cuh"
#include "eos_kernels.h"
#include "eosllm_cuda.h"

namespace {

enum : uint32_t {
  GV_U8 = 0, GV_I8 = 1, GV_U16 = 2, GV_I16 = 3, GV_U32 = 4, GV_I32 = 5, GV_F32 = 6, GV_BOOL = 7,
  GV_STRING = 8, GV_ARRAY = 9, GV_U64 = 10, GV_I64 = 11, GV_F64 = 12
};
enum : uint32_t { GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8, GGML_Q4_K = 12 };
constexpr uint32_t kMaxRank = 6;

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool err = false;
  template <typename T>
  T take() {
    T v{};
    if (err || (size_t)(end - p) < sizeof(T)) {
      err = true;
      return v;
    }
    memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  bool skip(uint64_t n) {
    if (err || (uint64_t)(end - p) < n) {
      err = true;
      return false;
    }
    p += n;
    return true;
  }
  std::string str() {
    const uint64_t n = take<uint64_t>();
    if (err || (uint64_t)(end - p) < n) {
      err = true;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p), (size_t)n);
    p += n;
    return s;
  }
};

uint32_t scalar_size(uint32_t t) {
  switch (t) {
    case GV_U8: case GV_I8: case GV_BOOL: return 1;
    case GV_U16: case GV_I16: return 2;
    case GV_U32: case GV_I32: case GV_F32: return 4;
    case GV_U64: case GV_I64: case GV_F64: return 8;
    default: return 0;
  }
}

struct Value {
  uint32_t type = 0;
  uint64_t bits = 0;  // scalar payload, little-endian, zero-extended
  std::string s;
};

struct TensorInfo {
  uint32_t rank = 0, ggml = 0;
  uint64_t dims[kMaxRank] = {};
  uint64_t offset = 0, bytes = 0;
  const uint8_t* data = nullptr;
};

// bytes of n elements of a GGML type; 0 for a partial block or an unknown type
uint64_t tensor_bytes(uint32_t ggml, uint64_t n) {
  switch (ggml) {
    case GGML_F32: return n * 4u;
    case GGML_F16: return n * 2u;
    case GGML_Q8_0: return n % 32u ? 0u : n / 32u * 34u;
    case GGML_Q4_K: return n % 256u ? 0u : n / 256u * 144u;
    default: return 0;
  }
}

int fail(int status, const char* msg) {
  eos::set_error_message(msg);
  return status;
}

}  // namespace

struct eosi_cuda_gguf {
  void* map = MAP_FAILED;
  size_t len = 0;
  std::unordered_map<std::string, Value> kv;
  std::unordered_map<std::string, TensorInfo> tensors;
  std::vector<const float*> attn_norm, ffn_norm;
  std::vector<const void*> wq, wk, wv, wo, wg, wu, wd;
  ~eosi_cuda_gguf() {
    if (map != MAP_FAILED) munmap(map, len);
  }

  // eos_model_meta_u64 (gguf.c:335-353): integer and bool types
  int meta_u64(const std::string& key, uint64_t* out) const {
    auto it = kv.find(key);
    if (it == kv.end()) return EOS_E_NOT_FOUND;
    const Value& v = it->second;
    switch (v.type) {
      case GV_U8: case GV_U16: case GV_U32: case GV_U64: case GV_BOOL: *out = v.bits; return EOS_OK;
      case GV_I8: *out = (uint64_t)(int64_t)(int8_t)v.bits; return EOS_OK;
      case GV_I16: *out = (uint64_t)(int64_t)(int16_t)v.bits; return EOS_OK;
      case GV_I32: *out = (uint64_t)(int64_t)(int32_t)v.bits; return EOS_OK;
      case GV_I64: *out = v.bits; return EOS_OK;
      default: return EOS_E_INVALID_ARG;
    }
  }
  // eos_model_meta_f32 (gguf.c:355-362): F32 values only
  int meta_f32(const std::string& key, float* out) const {
    auto it = kv.find(key);
    if (it == kv.end()) return EOS_E_NOT_FOUND;
    if (it->second.type != GV_F32) return EOS_E_INVALID_ARG;
    uint32_t b = (uint32_t)it->second.bits;
    memcpy(out, &b, 4);
    return EOS_OK;
  }
  const TensorInfo* tensor(const std::string& name) const {
    auto it = tensors.find(name);
    return it == tensors.end() ? nullptr : &it->second;
  }

  int parse();
  int describe(uint32_t max_ctx, eosi_cuda_llama_t* d);
};

int eosi_cuda_gguf::parse() {
  Cursor c{static_cast<const uint8_t*>(map), static_cast<const uint8_t*>(map) + len};
  const uint32_t magic = c.take<uint32_t>(), version = c.take<uint32_t>();
  const uint64_t n_tensors = c.take<uint64_t>(), n_kv = c.take<uint64_t>();
  if (c.err || magic != 0x46554747u || version != 3u)
    return fail(EOS_E_FORMAT, "gguf: bad magic or unsupported version (expected GGUF v3)");
  uint32_t alignment = 32;
  for (uint64_t i = 0; i < n_kv && !c.err; ++i) {
    std::string key = c.str();
    Value v;
    v.type = c.take<uint32_t>();
    if (c.err) break;
    if (v.type == GV_STRING) {
      v.s = c.str();
    } else if (v.type == GV_ARRAY) {
      const uint32_t et = c.take<uint32_t>();
      const uint64_t count = c.take<uint64_t>();
      v.bits = count;
      if (et == GV_STRING) {
        for (uint64_t j = 0; j < count && !c.err; ++j) {
          const uint64_t n = c.take<uint64_t>();
          c.skip(n);
        }
      } else if (scalar_size(et) != 0) {
        if (count > (uint64_t)(c.end - c.p) / scalar_size(et)) c.err = true;
        else c.skip(count * scalar_size(et));
      } else {
        return fail(EOS_E_FORMAT, "gguf: unsupported array element type");
      }
    } else if (scalar_size(v.type) != 0) {
      const uint32_t n = scalar_size(v.type);
      if ((size_t)(c.end - c.p) < n) c.err = true;
      else {
        memcpy(&v.bits, c.p, n);
        c.p += n;
      }
    } else {
      return fail(EOS_E_FORMAT, "gguf: unknown metadata value type");
    }
    if (key == "general.alignment") {  // gguf.c:579-590
      uint64_t a = 0;
      kv[key] = v;
      if (meta_u64(key, &a) == EOS_OK) {
        if (a == 0 || (a & (a - 1)) != 0 || a > (1u << 30))
          return fail(EOS_E_FORMAT, "gguf: general.alignment is not power-of-two");
        alignment = (uint32_t)a;
      }
    }
    kv[key] = std::move(v);
  }
  if (c.err) return fail(EOS_E_FORMAT, "gguf: truncated metadata");
  std::vector<std::pair<std::string, TensorInfo>> order;
  for (uint64_t i = 0; i < n_tensors && !c.err; ++i) {
    std::string name = c.str();
    TensorInfo t;
    t.rank = c.take<uint32_t>();
    if (c.err) break;
    if (t.rank == 0 || t.rank > kMaxRank) return fail(EOS_E_FORMAT, "gguf: tensor has rank 0 or > 6");
    uint64_t elems = 1;
    for (uint32_t j = 0; j < t.rank; ++j) {
      const uint64_t dd = c.take<uint64_t>();
      if (c.err) break;
      if (dd == 0 || dd > 0xFFFFFFFFull) return fail(EOS_E_FORMAT, "gguf: tensor has zero or oversized dim");
      if (elems > ~0ull / dd) return fail(EOS_E_FORMAT, "gguf: tensor element count overflows u64");
      t.dims[j] = dd;
      elems *= dd;
    }
    t.ggml = c.take<uint32_t>();
    if (c.err) break;
    if (t.ggml != GGML_F32 && t.ggml != GGML_F16 && t.ggml != GGML_Q8_0 && t.ggml != GGML_Q4_K)
      return fail(EOS_E_UNSUPPORTED, "gguf: tensor uses unsupported dtype");
    t.bytes = tensor_bytes(t.ggml, elems);
    if (t.bytes == 0) return fail(EOS_E_FORMAT, "gguf: tensor element count not divisible by block size");
    t.offset = c.take<uint64_t>();
    order.emplace_back(std::move(name), t);
  }
  if (c.err) return fail(EOS_E_FORMAT, "gguf: truncated tensor infos");
  const size_t data_off = (size_t)(c.p - static_cast<const uint8_t*>(map));
  if (data_off > ~(size_t)0 - (alignment - 1u)) return fail(EOS_E_FORMAT, "gguf: tensor data offset overflows");
  const size_t aligned = (data_off + alignment - 1u) & ~((size_t)alignment - 1u);
  if (aligned > len) return fail(EOS_E_FORMAT, "gguf: aligned data offset is past EOF");
  const size_t limit = len - aligned;
  for (auto& [name, t] : order) {
    if (t.offset > limit || t.bytes > limit - t.offset) return fail(EOS_E_FORMAT, "gguf: tensor data extends past EOF");
    t.data = static_cast<const uint8_t*>(map) + aligned + t.offset;
    tensors[name] = t;
  }
  return EOS_OK;
}

int eosi_cuda_gguf::describe(uint32_t max_ctx, eosi_cuda_llama_t* d) {
  auto ait = kv.find("general.architecture");
  if (ait == kv.end() || ait->second.type != GV_STRING)
    return fail(EOS_E_FORMAT, "gguf: general.architecture missing");
  const std::string arch = ait->second.s + ".";
  uint64_t v = 0;
  int s;
  memset(d, 0, sizeof(*d));
  if ((s = meta_u64(arch + "embedding_length", &v)) != EOS_OK) return fail(s, "gguf: embedding_length missing");
  d->n_embd = (uint32_t)v;
  if ((s = meta_u64(arch + "block_count", &v)) != EOS_OK) return fail(s, "gguf: block_count missing");
  d->n_layer = (uint32_t)v;
  if ((s = meta_u64(arch + "attention.head_count", &v)) != EOS_OK) return fail(s, "gguf: head_count missing");
  d->n_head = (uint32_t)v;
  d->n_kv_head = meta_u64(arch + "attention.head_count_kv", &v) == EOS_OK ? (uint32_t)v : d->n_head;
  if ((s = meta_u64(arch + "feed_forward_length", &v)) != EOS_OK) return fail(s, "gguf: feed_forward_length missing");
  d->n_ff = (uint32_t)v;
  if ((s = meta_u64(arch + "context_length", &v)) != EOS_OK) return fail(s, "gguf: context_length missing");
  d->max_ctx = (uint32_t)v;
  if (max_ctx > 0 && max_ctx < d->max_ctx) d->max_ctx = max_ctx;
  if (d->n_head == 0 || d->n_kv_head == 0) return fail(EOS_E_FORMAT, "gguf: zero head count");
  if (meta_f32(arch + "rope.freq_base", &d->rope_base) != EOS_OK) d->rope_base = 10000.0f;
  if (meta_f32(arch + "attention.layer_norm_rms_epsilon", &d->rms_eps) != EOS_OK) d->rms_eps = 1e-5f;

  const TensorInfo* emb = tensor("token_embd.weight");
  const TensorInfo* onorm = tensor("output_norm.weight");
  const TensorInfo* out = tensor("output.weight");
  if (emb == nullptr || onorm == nullptr) return fail(EOS_E_FORMAT, "gguf: token_embd or output_norm missing");
  d->n_vocab = (uint32_t)(emb->rank > 1 ? emb->dims[1] : emb->dims[0]);
  const uint32_t E = d->n_embd, hd = d->n_head ? E / d->n_head : 0, kvd = hd * d->n_kv_head;
  if (emb->ggml != GGML_F16) return fail(EOS_E_UNSUPPORTED, "gguf: token embeddings must be F16 for the device decoder");
  if (out == nullptr) return fail(EOS_E_UNSUPPORTED, "gguf: tied output (no output.weight) is not supported");
  auto qdt = [](uint32_t g) { return g == GGML_Q4_K ? EOS_DT_Q4_K : (g == GGML_Q8_0 ? EOS_DT_Q8_0 : -1); };
  auto is2d = [](const TensorInfo* t, uint64_t in, uint64_t o) {
    return t != nullptr && t->rank == 2 && t->dims[0] == in && t->dims[1] == o;
  };
  auto is1d = [](const TensorInfo* t, uint64_t n) {
    return t != nullptr && t->ggml == GGML_F32 && t->rank == 1 && t->dims[0] == n;
  };
  if (!is2d(emb, E, d->n_vocab) || !is1d(onorm, E) || !is2d(out, E, d->n_vocab))
    return fail(EOS_E_FORMAT, "gguf: embedding / output shapes do not match embedding_length");
  d->out_dtype = qdt(out->ggml);
  if (d->out_dtype < 0) return fail(EOS_E_UNSUPPORTED, "gguf: output.weight must be Q4_K or Q8_0");
  d->tok_embd = reinterpret_cast<const uint16_t*>(emb->data);
  d->output_norm = reinterpret_cast<const float*>(onorm->data);
  d->output_w = out->data;
  attn_norm.assign(d->n_layer, nullptr);
  ffn_norm.assign(d->n_layer, nullptr);
  for (auto* vec : {&wq, &wk, &wv, &wo, &wg, &wu, &wd}) vec->assign(d->n_layer, nullptr);
  int wdt = -1;
  for (uint32_t L = 0; L < d->n_layer; ++L) {
    const std::string b = "blk." + std::to_string(L) + ".";
    const TensorInfo* t[9] = {tensor(b + "attn_norm.weight"), tensor(b + "attn_q.weight"),
                              tensor(b + "attn_k.weight"), tensor(b + "attn_v.weight"),
                              tensor(b + "attn_output.weight"), tensor(b + "ffn_norm.weight"),
                              tensor(b + "ffn_gate.weight"), tensor(b + "ffn_up.weight"),
                              tensor(b + "ffn_down.weight")};
    for (const TensorInfo* x : t)
      if (x == nullptr) return fail(EOS_E_FORMAT, "gguf: a layer tensor is missing");
    if (!is1d(t[0], E) || !is2d(t[1], E, E) || !is2d(t[2], E, kvd) || !is2d(t[3], E, kvd) ||
        !is2d(t[4], E, E) || !is1d(t[5], E) || !is2d(t[6], E, d->n_ff) || !is2d(t[7], E, d->n_ff) ||
        !is2d(t[8], d->n_ff, E))
      return fail(EOS_E_FORMAT, "gguf: a layer tensor's shape does not match the hyper-parameters");
    for (int i : {1, 2, 3, 4, 6, 7, 8}) {
      const int q = qdt(t[i]->ggml);
      if (q < 0 || (wdt >= 0 && q != wdt))
        return fail(EOS_E_UNSUPPORTED, "gguf: block linears must all be Q4_K or all Q8_0");
      wdt = q;
    }
    attn_norm[L] = reinterpret_cast<const float*>(t[0]->data);
    wq[L] = t[1]->data;
    wk[L] = t[2]->data;
    wv[L] = t[3]->data;
    wo[L] = t[4]->data;
    ffn_norm[L] = reinterpret_cast<const float*>(t[5]->data);
    wg[L] = t[6]->data;
    wu[L] = t[7]->data;
    wd[L] = t[8]->data;
  }
  d->wdtype = wdt < 0 ? d->out_dtype : wdt;
  d->weights_on_device = 0;
  d->attn_norm = attn_norm.data();
  d->ffn_norm = ffn_norm.data();
  d->wq = wq.data();
  d->wk = wk.data();
  d->wv = wv.data();
  d->wo = wo.data();
  d->wg = wg.data();
  d->wu = wu.data();
  d->wd = wd.data();
  return EOS_OK;
}

extern "C" {

EOSLLM_CUDA_API int eosi_cuda_gguf_map(const char* path, uint32_t max_ctx, eosi_cuda_gguf_t** out,
                                       eosi_cuda_llama_t* desc) {
  if (path == nullptr || out == nullptr || desc == nullptr) return EOS_E_INVALID_ARG;
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(EOS_E_IO, "gguf: cannot open the file");
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    return fail(EOS_E_FORMAT, "gguf: empty file");
  }
  eosi_cuda_gguf_t* g = new (std::nothrow) eosi_cuda_gguf_t();
  if (g == nullptr) {
    close(fd);
    return EOS_E_OUT_OF_MEMORY;
  }
  g->len = (size_t)st.st_size;
  g->map = mmap(nullptr, g->len, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (g->map == MAP_FAILED) {
    delete g;
    return fail(EOS_E_IO, "gguf: cannot map the file");
  }
  int s = g->parse();
  if (s == EOS_OK) s = g->describe(max_ctx, desc);
  if (s != EOS_OK) {
    delete g;
    return s;
  }
  *out = g;
  return EOS_OK;
}

EOSLLM_CUDA_API void eosi_cuda_gguf_unmap(eosi_cuda_gguf_t* g) { delete g; }

EOSLLM_CUDA_API int eosi_cuda_text_open_gguf(const char* path, uint32_t max_ctx, int device, int rank, int world,
                                             eosi_cuda_text_t** out) {
  if (out == nullptr) return EOS_E_INVALID_ARG;
  *out = nullptr;
  eosi_cuda_gguf_t* g = nullptr;
  eosi_cuda_llama_t d;
  int s = eosi_cuda_gguf_map(path, max_ctx, &g, &d);
  if (s != EOS_OK) return s;
  s = eosi_cuda_text_open(&d, device, rank, world, out);  // copies this rank's slices, synchronously
  eosi_cuda_gguf_unmap(g);
  return s;
}

}  // extern "C"
