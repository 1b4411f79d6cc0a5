// safetensors.cpp -- reader for quantize.cu's INT8 checkpoint format.
//
// File layout (safetensors.h:36-113 of the reference): 8-byte little-endian
// header length, a JSON object {name: {"dtype", "shape", "data_offsets"}},
// then the raw tensor bytes.  A ".json" path is read as a sharded index
// ({"weight_map": {name: file}}, safetensors.h:115-150).  INT8 linears are
// "<name>" I8 [N,K] + "<name>.__scales__" F32 [N]; biases, norm weights and the
// boundary layers are BF16 (quantize.cu:121-137, 467-477).  A BF16 weight
// found where an INT8 linear is expected is quantized at load time with the
// product's bit-exact weight quantizer, like TransformerWeights::load's
// fallback (transformer.h:193-199).
//
// Tensors are read into pinned host memory in 64 MB pieces and copied to
// per-tensor device buffers; qi_model_create then builds the kernel layout.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/qwen_image_b200.h"
#include "qi_internal.h"

namespace {

struct TInfo {
  std::string file, dtype;
  std::vector<long long> shape;
  size_t begin = 0, end = 0, data_start = 0;
};

// Minimal JSON reader for safetensors headers and index files.
struct Json {
  const char* p;
  const char* e;
  bool ok = true;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  std::string str() {
    ws();
    std::string s;
    if (p >= e || *p != '"') {
      ok = false;
      return s;
    }
    ++p;
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) {
        ++p;
        char c = *p;
        s.push_back(c == 'n' ? '\n' : c == 't' ? '\t' : c);
      } else {
        s.push_back(*p);
      }
      ++p;
    }
    if (p < e) ++p;
    return s;
  }
  long long num() {
    ws();
    char* end = nullptr;
    long long v = strtoll(p, &end, 10);
    if (end == p) ok = false;
    p = end;
    // skip fractional parts if any
    while (p < e && (*p == '.' || *p == 'e' || *p == 'E' || *p == '+' || *p == '-' || (*p >= '0' && *p <= '9'))) ++p;
    return v;
  }
  void skip() {
    ws();
    if (p >= e) {
      ok = false;
      return;
    }
    if (*p == '"') {
      str();
    } else if (*p == '{') {
      ++p;
      if (eat('}')) return;
      do {
        str();
        if (!eat(':')) {
          ok = false;
          return;
        }
        skip();
      } while (ok && eat(','));
      if (!eat('}')) ok = false;
    } else if (*p == '[') {
      ++p;
      if (eat(']')) return;
      do skip();
      while (ok && eat(','));
      if (!eat(']')) ok = false;
    } else if (!strncmp(p, "true", 4) || !strncmp(p, "null", 4)) {
      p += 4;
    } else if (!strncmp(p, "false", 5)) {
      p += 5;
    } else {
      num();
    }
  }
};

bool read_file(const std::string& path, std::string& out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  out.resize(static_cast<size_t>(n));
  bool ok = fread(&out[0], 1, static_cast<size_t>(n), f) == static_cast<size_t>(n);
  fclose(f);
  return ok;
}

bool parse_header(const std::string& path, std::map<std::string, TInfo>& infos) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  uint64_t hlen = 0;
  if (fread(&hlen, 8, 1, f) != 1 || hlen > (1ull << 30)) {
    fclose(f);
    return false;
  }
  std::string h(hlen, '\0');
  bool ok = fread(&h[0], 1, hlen, f) == hlen;
  fclose(f);
  if (!ok) return false;
  Json j{h.data(), h.data() + h.size()};
  if (!j.eat('{')) return false;
  if (j.eat('}')) return true;
  do {
    std::string key = j.str();
    if (!j.eat(':')) return false;
    if (key == "__metadata__") {
      j.skip();
      continue;
    }
    TInfo t;
    t.file = path;
    t.data_start = 8 + hlen;
    if (!j.eat('{')) return false;
    do {
      std::string f2 = j.str();
      if (!j.eat(':')) return false;
      if (f2 == "dtype") {
        t.dtype = j.str();
      } else if (f2 == "shape") {
        if (!j.eat('[')) return false;
        if (!j.eat(']')) {
          do t.shape.push_back(j.num());
          while (j.eat(','));
          if (!j.eat(']')) return false;
        }
      } else if (f2 == "data_offsets") {
        if (!j.eat('[')) return false;
        t.begin = static_cast<size_t>(j.num());
        j.eat(',');
        t.end = static_cast<size_t>(j.num());
        if (!j.eat(']')) return false;
      } else {
        j.skip();
      }
    } while (j.ok && j.eat(','));
    if (!j.eat('}')) return false;
    infos[key] = t;
  } while (j.ok && j.eat(','));
  return j.ok;
}

bool parse_index(const std::string& path, std::map<std::string, TInfo>& infos) {
  std::string text;
  if (!read_file(path, text)) return false;
  std::string dir = path.substr(0, path.find_last_of('/') + 1);
  Json j{text.data(), text.data() + text.size()};
  std::map<std::string, bool> files;
  if (!j.eat('{')) return false;
  do {
    std::string key = j.str();
    if (!j.eat(':')) return false;
    if (key != "weight_map") {
      j.skip();
      continue;
    }
    if (!j.eat('{')) return false;
    if (!j.eat('}')) {
      do {
        j.str();
        if (!j.eat(':')) return false;
        files[j.str()] = true;
      } while (j.ok && j.eat(','));
      if (!j.eat('}')) return false;
    }
  } while (j.ok && j.eat(','));
  for (auto& kv : files)
    if (!parse_header(dir + kv.first, infos)) return false;
  return j.ok;
}

size_t dtype_bytes(const std::string& d) {
  if (d == "I8" || d == "U8") return 1;
  if (d == "BF16" || d == "F16") return 2;
  if (d == "F32" || d == "I32") return 4;
  return 0;
}

struct Loader {
  std::map<std::string, TInfo> infos;
  std::vector<void*> dev;  // temporary device tensors
  void* pinned = nullptr;
  size_t pinned_cap = 0;
  ~Loader() {
    for (void* p : dev) cudaFree(p);
    if (pinned) cudaFreeHost(pinned);
  }
  const TInfo* find(const std::string& n) const {
    auto it = infos.find(n);
    return it == infos.end() ? nullptr : &it->second;
  }
  // Uploads tensor `n` (checks dtype and element count); returns device ptr.
  void* load(const std::string& n, const char* dtype, long long numel, int* st) {
    const TInfo* t = find(n);
    if (!t || t->dtype != dtype) {
      *st = QI_ERR_IO;
      return nullptr;
    }
    long long cnt = 1;
    for (long long d : t->shape) cnt *= d;
    const size_t bytes = t->end - t->begin;
    if (cnt != numel || bytes != static_cast<size_t>(numel) * dtype_bytes(t->dtype)) {
      *st = QI_ERR_IO;
      return nullptr;
    }
    void* d = nullptr;
    if (qi::dev_malloc(&d, bytes < 16 ? 16 : bytes) != cudaSuccess) {
      *st = QI_ERR_OOM;
      return nullptr;
    }
    dev.push_back(d);
    const size_t chunk = 64ull << 20;
    if (!pinned) {
      if (qi::host_malloc_pinned(&pinned, chunk) != cudaSuccess) {
        *st = QI_ERR_OOM;
        return nullptr;
      }
      pinned_cap = chunk;
    }
    FILE* f = fopen(t->file.c_str(), "rb");
    if (!f) {
      *st = QI_ERR_IO;
      return nullptr;
    }
    fseek(f, static_cast<long>(t->data_start + t->begin), SEEK_SET);
    for (size_t off = 0; off < bytes; off += chunk) {
      const size_t n2 = bytes - off < chunk ? bytes - off : chunk;
      if (fread(pinned, 1, n2, f) != n2) {
        fclose(f);
        *st = QI_ERR_IO;
        return nullptr;
      }
      if (cudaMemcpy(static_cast<char*>(d) + off, pinned, n2, cudaMemcpyHostToDevice) != cudaSuccess) {
        fclose(f);
        *st = QI_ERR_CUDA;
        return nullptr;
      }
    }
    fclose(f);
    return d;
  }
  // INT8 linear: codes + scales, or a BF16 weight quantized at load time.
  int load_int8(const std::string& w, int N, int K, void** codes, void** scales) {
    int st = QI_OK;
    const TInfo* t = find(w);
    if (!t) return QI_ERR_IO;
    if (t->dtype == "I8") {
      *codes = load(w, "I8", static_cast<long long>(N) * K, &st);
      if (st) return st;
      *scales = load(w + ".__scales__", "F32", N, &st);
      return st;
    }
    if (t->dtype != "BF16") return QI_ERR_UNSUPPORTED;
    void* wb = load(w, "BF16", static_cast<long long>(N) * K, &st);
    if (st) return st;
    void *c = nullptr, *s = nullptr;
    if (qi::dev_malloc(reinterpret_cast<void**>(&c), static_cast<size_t>(N) * K) != cudaSuccess) return QI_ERR_OOM;
    dev.push_back(c);
    if (qi::dev_malloc(reinterpret_cast<void**>(&s), static_cast<size_t>(N) * 4) != cudaSuccess) return QI_ERR_OOM;
    dev.push_back(s);
    st = qi_quantize_weight(wb, N, K, static_cast<int8_t*>(c), static_cast<float*>(s), nullptr);
    if (st) return st;
    *codes = c;
    *scales = s;
    return cudaDeviceSynchronize() == cudaSuccess ? QI_OK : QI_ERR_CUDA;
  }
};

}  // namespace

extern "C" int qi_model_load_safetensors(qi_ctx* ctx, const char* path, qi_model** out) {
  if (!ctx || !path || !out) return QI_ERR_ARG;
  Loader L;
  std::string p(path);
  const bool index = p.size() > 5 && p.substr(p.size() - 5) == ".json";
  if (!(index ? parse_index(p, L.infos) : parse_header(p, L.infos))) return QI_ERR_IO;
  int nblocks = 0;
  while (L.find("transformer_blocks." + std::to_string(nblocks) + ".attn.to_q.weight")) ++nblocks;
  if (nblocks == 0) return QI_ERR_IO;
  int st = QI_OK;
  std::vector<const void*> g(QI_G_COUNT, nullptr);
  void *c = nullptr, *s = nullptr;
  const std::string te = "time_text_embed.timestep_embedder.";
  if ((st = L.load_int8(te + "linear_1.weight", 3072, 256, &c, &s))) return st;
  g[QI_G_T1_W] = c;
  g[QI_G_T1_S] = s;
  if ((st = L.load_int8(te + "linear_2.weight", 3072, 3072, &c, &s))) return st;
  g[QI_G_T2_W] = c;
  g[QI_G_T2_S] = s;
  struct B16 {
    int idx;
    const char* name;
    long long n;
  };
  const B16 bf[] = {{QI_G_T1_B, "time_text_embed.timestep_embedder.linear_1.bias", 3072},
                    {QI_G_T2_B, "time_text_embed.timestep_embedder.linear_2.bias", 3072},
                    {QI_G_TXT_NORM, "txt_norm.weight", 3584},
                    {QI_G_IMG_IN_W, "img_in.weight", 3072LL * 64},
                    {QI_G_IMG_IN_B, "img_in.bias", 3072},
                    {QI_G_TXT_IN_W, "txt_in.weight", 3072LL * 3584},
                    {QI_G_TXT_IN_B, "txt_in.bias", 3072},
                    {QI_G_NORM_OUT_W, "norm_out.linear.weight", 6144LL * 3072},
                    {QI_G_NORM_OUT_B, "norm_out.linear.bias", 6144},
                    {QI_G_PROJ_OUT_W, "proj_out.weight", 64LL * 3072},
                    {QI_G_PROJ_OUT_B, "proj_out.bias", 64}};
  for (const B16& b : bf) {
    g[b.idx] = L.load(b.name, "BF16", b.n, &st);
    if (st) return st == QI_ERR_IO ? QI_ERR_UNSUPPORTED : st;  // INT8 boundary layers are not supported
  }
  static const char* lnames[QI_L_COUNT] = {"img_mod.1",        "txt_mod.1",        "attn.to_q",
                                           "attn.to_k",        "attn.to_v",        "attn.add_q_proj",
                                           "attn.add_k_proj",  "attn.add_v_proj",  "attn.to_out.0",
                                           "attn.to_add_out",  "img_mlp.net.0.proj", "img_mlp.net.2",
                                           "txt_mlp.net.0.proj", "txt_mlp.net.2"};
  static const int ldims[QI_L_COUNT][2] = {{18432, 3072}, {18432, 3072}, {3072, 3072}, {3072, 3072},
                                           {3072, 3072},  {3072, 3072},  {3072, 3072}, {3072, 3072},
                                           {3072, 3072},  {3072, 3072},  {12288, 3072}, {3072, 12288},
                                           {12288, 3072}, {3072, 12288}};
  static const char* nnames[4] = {"attn.norm_q.weight", "attn.norm_k.weight", "attn.norm_added_q.weight",
                                  "attn.norm_added_k.weight"};
  std::vector<std::vector<const void*>> blocks(nblocks, std::vector<const void*>(QI_B_COUNT, nullptr));
  std::vector<const void* const*> bt(nblocks);
  for (int i = 0; i < nblocks; ++i) {
    const std::string pre = "transformer_blocks." + std::to_string(i) + ".";
    for (int l = 0; l < QI_L_COUNT; ++l) {
      if ((st = L.load_int8(pre + lnames[l] + ".weight", ldims[l][0], ldims[l][1], &c, &s))) return st;
      blocks[i][3 * l] = c;
      blocks[i][3 * l + 1] = s;
      blocks[i][3 * l + 2] = L.load(pre + lnames[l] + ".bias", "BF16", ldims[l][0], &st);
      if (st) return st;
    }
    for (int k = 0; k < 4; ++k) {
      blocks[i][QI_B_NORM_Q + k] = L.load(pre + nnames[k], "BF16", 128, &st);
      if (st) return st;
    }
    bt[i] = blocks[i].data();
  }
  return qi_model_create(ctx, nblocks, g.data(), bt.data(), out);
}
