// Whole-path sample_actions engine (svla_engine_* in svla.h): loads a packed-weights safetensors file into
// one device arena, sizes the activation buffers for max_batch samples, and runs the quantized call as a
// list of libsvla launches per batch size, recorded as a CUDA graph after its first run.  The launch order
// and every descriptor follow the Python runner (smolvla_mujoco_libero_b200/model.py, SmolVLARunner._build),
// so the two give bit-identical actions for the same file and inputs.
//
// Host code only; compiled into libsvla.so next to svla.cu.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/svla.h"

namespace svla {
int32_t set_error(int32_t code, const std::string& msg);  // svla.cu

namespace engine_impl {

std::string fmt(const char* f, ...) __attribute__((format(printf, 1, 2)));
std::string fmt(const char* f, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, f);
  vsnprintf(buf, sizeof(buf), f, ap);
  va_end(ap);
  return buf;
}

// ----------------------------------------------------------------------------------------------- JSON
// The subset of JSON the safetensors header and the packed metadata use (RFC 8259 values; numbers as
// double, exact for the integers here, which stay below 2^53).
struct Json {
  enum Type { kNull, kBool, kNum, kStr, kArr, kObj } type = kNull;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;

  const Json* get(const std::string& key) const {
    if (type != kObj) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
};

class JsonParser {
 public:
  JsonParser(const char* s, size_t n) : p_(s), end_(s + n) {}

  bool parse(Json* out, std::string* err) {
    ws();
    if (!value(out, 0)) {
      *err = err_.empty() ? "malformed JSON" : err_;
      return false;
    }
    ws();
    if (p_ != end_) {
      *err = "trailing characters after the JSON value";
      return false;
    }
    return true;
  }

 private:
  const char* p_;
  const char* end_;
  std::string err_;

  void ws() {
    while (p_ < end_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
  }
  bool fail(const char* what) {
    if (err_.empty()) err_ = what;
    return false;
  }
  bool literal(const char* word) {
    const size_t n = std::strlen(word);
    if (static_cast<size_t>(end_ - p_) < n || std::memcmp(p_, word, n) != 0) return fail("bad literal");
    p_ += n;
    return true;
  }
  static void utf8(uint32_t c, std::string* s) {
    if (c < 0x80) {
      s->push_back(static_cast<char>(c));
    } else if (c < 0x800) {
      s->push_back(static_cast<char>(0xC0 | (c >> 6)));
      s->push_back(static_cast<char>(0x80 | (c & 0x3F)));
    } else if (c < 0x10000) {
      s->push_back(static_cast<char>(0xE0 | (c >> 12)));
      s->push_back(static_cast<char>(0x80 | ((c >> 6) & 0x3F)));
      s->push_back(static_cast<char>(0x80 | (c & 0x3F)));
    } else {
      s->push_back(static_cast<char>(0xF0 | (c >> 18)));
      s->push_back(static_cast<char>(0x80 | ((c >> 12) & 0x3F)));
      s->push_back(static_cast<char>(0x80 | ((c >> 6) & 0x3F)));
      s->push_back(static_cast<char>(0x80 | (c & 0x3F)));
    }
  }
  bool hex4(uint32_t* v) {
    if (end_ - p_ < 4) return fail("short \\u escape");
    uint32_t r = 0;
    for (int i = 0; i < 4; ++i) {
      const char c = *p_++;
      r <<= 4;
      if (c >= '0' && c <= '9') r |= static_cast<uint32_t>(c - '0');
      else if (c >= 'a' && c <= 'f') r |= static_cast<uint32_t>(c - 'a' + 10);
      else if (c >= 'A' && c <= 'F') r |= static_cast<uint32_t>(c - 'A' + 10);
      else return fail("bad \\u escape");
    }
    *v = r;
    return true;
  }
  bool string(std::string* s) {
    if (p_ >= end_ || *p_ != '"') return fail("expected a string");
    ++p_;
    while (p_ < end_ && *p_ != '"') {
      const char c = *p_++;
      if (static_cast<unsigned char>(c) < 0x20) return fail("control character in a string");
      if (c != '\\') {
        s->push_back(c);
        continue;
      }
      if (p_ >= end_) return fail("unterminated escape");
      const char e = *p_++;
      switch (e) {
        case '"': s->push_back('"'); break;
        case '\\': s->push_back('\\'); break;
        case '/': s->push_back('/'); break;
        case 'b': s->push_back('\b'); break;
        case 'f': s->push_back('\f'); break;
        case 'n': s->push_back('\n'); break;
        case 'r': s->push_back('\r'); break;
        case 't': s->push_back('\t'); break;
        case 'u': {
          uint32_t c1 = 0;
          if (!hex4(&c1)) return false;
          if (c1 >= 0xD800 && c1 < 0xDC00) {  // surrogate pair
            uint32_t c2 = 0;
            if (end_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return fail("lone surrogate");
            p_ += 2;
            if (!hex4(&c2) || c2 < 0xDC00 || c2 >= 0xE000) return fail("bad surrogate pair");
            c1 = 0x10000 + ((c1 - 0xD800) << 10) + (c2 - 0xDC00);
          }
          utf8(c1, s);
          break;
        }
        default: return fail("bad escape");
      }
    }
    if (p_ >= end_) return fail("unterminated string");
    ++p_;
    return true;
  }
  bool number(double* v) {
    const char* start = p_;
    if (p_ < end_ && (*p_ == '-' || *p_ == '+')) ++p_;
    while (p_ < end_ && ((*p_ >= '0' && *p_ <= '9') || *p_ == '.' || *p_ == 'e' || *p_ == 'E' || *p_ == '-' ||
                         *p_ == '+'))
      ++p_;
    // Python's json module writes non-finite floats as these words
    if (p_ == start || (p_ == start + 1 && (*start == '-' || *start == '+'))) {
      for (const char* w : {"Infinity", "NaN"}) {
        const size_t n = std::strlen(w);
        if (static_cast<size_t>(end_ - p_) >= n && std::memcmp(p_, w, n) == 0) {
          p_ += n;
          const double x = (w[0] == 'N') ? NAN : INFINITY;
          *v = (*start == '-') ? -x : x;
          return true;
        }
      }
      return fail("expected a number");
    }
    const std::string tok(start, p_);
    char* endp = nullptr;
    *v = std::strtod(tok.c_str(), &endp);
    if (endp != tok.c_str() + tok.size()) return fail("bad number");
    return true;
  }
  bool value(Json* v, int depth) {
    if (depth > 32) return fail("JSON nested too deeply");
    ws();
    if (p_ >= end_) return fail("unexpected end of JSON");
    const char c = *p_;
    if (c == '{') {
      ++p_;
      v->type = Json::kObj;
      ws();
      if (p_ < end_ && *p_ == '}') {
        ++p_;
        return true;
      }
      for (;;) {
        ws();
        std::string key;
        if (!string(&key)) return false;
        ws();
        if (p_ >= end_ || *p_ != ':') return fail("expected ':'");
        ++p_;
        Json item;
        if (!value(&item, depth + 1)) return false;
        v->obj.emplace_back(std::move(key), std::move(item));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == '}') {
          ++p_;
          return true;
        }
        return fail("expected ',' or '}'");
      }
    }
    if (c == '[') {
      ++p_;
      v->type = Json::kArr;
      ws();
      if (p_ < end_ && *p_ == ']') {
        ++p_;
        return true;
      }
      for (;;) {
        Json item;
        if (!value(&item, depth + 1)) return false;
        v->arr.push_back(std::move(item));
        ws();
        if (p_ < end_ && *p_ == ',') {
          ++p_;
          continue;
        }
        if (p_ < end_ && *p_ == ']') {
          ++p_;
          return true;
        }
        return fail("expected ',' or ']'");
      }
    }
    if (c == '"') {
      v->type = Json::kStr;
      return string(&v->str);
    }
    if (c == 't') {
      v->type = Json::kBool;
      v->b = true;
      return literal("true");
    }
    if (c == 'f') {
      v->type = Json::kBool;
      return literal("false");
    }
    if (c == 'n') {
      v->type = Json::kNull;
      return literal("null");
    }
    v->type = Json::kNum;
    return number(&v->num);
  }
};

bool parse_json(const std::string& text, Json* out, std::string* err) {
  return JsonParser(text.data(), text.size()).parse(out, err);
}

// ----------------------------------------------------------------------------------------------- config
// The architecture fields of SmolVLAConfig (smolvla_mujoco_libero_b200/config.py) that the call needs.
struct Cfg {
  int image_size, patch, channels, vis_hidden, vis_layers, vis_heads, vis_mlp, scale_factor, n_cams;
  double vis_eps;
  int hidden, text_layers, heads, kv_heads, head_dim, mlp, vocab;
  double rms_eps, rope_wavelength;
  int expert_hidden, expert_layers, expert_mlp, self_attn_every_n_layers;
  int n_lang, max_state_dim, max_action_dim, action_dim, chunk, num_steps;

  int grid() const { return image_size / patch; }
  int n_patches() const { return grid() * grid(); }
  int n_img_tokens() const { return n_patches() / (scale_factor * scale_factor); }
  int prefix_len() const { return n_cams * n_img_tokens() + n_lang + 1; }
  int kv_dim() const { return kv_heads * head_dim; }
  int q_dim() const { return heads * head_dim; }
  // lerobot SmolVLMWithExpertModel.forward: cross-attention unless layer % n == 0
  bool is_cross(int layer) const {
    return !(self_attn_every_n_layers > 0 && layer % self_attn_every_n_layers == 0);
  }
};

bool read_cfg(const Json& j, Cfg* c, std::string* err) {
  auto num = [&](const char* key, double* out) {
    const Json* v = j.get(key);
    if (!v || v->type != Json::kNum) {
      *err = fmt("config field %s missing or not a number", key);
      return false;
    }
    *out = v->num;
    return true;
  };
  auto integer = [&](const char* key, int* out) {
    double v = 0;
    if (!num(key, &v)) return false;
    if (v != std::floor(v) || v < 0 || v > 1e9) {
      *err = fmt("config field %s is not a non-negative integer", key);
      return false;
    }
    *out = static_cast<int>(v);
    return true;
  };
  const bool ok =
      integer("image_size", &c->image_size) && integer("patch", &c->patch) && integer("channels", &c->channels) &&
      integer("vis_hidden", &c->vis_hidden) && integer("vis_layers", &c->vis_layers) &&
      integer("vis_heads", &c->vis_heads) && integer("vis_mlp", &c->vis_mlp) && num("vis_eps", &c->vis_eps) &&
      integer("scale_factor", &c->scale_factor) && integer("n_cams", &c->n_cams) && integer("hidden", &c->hidden) &&
      integer("text_layers", &c->text_layers) && integer("heads", &c->heads) && integer("kv_heads", &c->kv_heads) &&
      integer("head_dim", &c->head_dim) && integer("mlp", &c->mlp) && num("rms_eps", &c->rms_eps) &&
      integer("vocab", &c->vocab) && num("rope_wavelength", &c->rope_wavelength) &&
      integer("expert_hidden", &c->expert_hidden) && integer("expert_layers", &c->expert_layers) &&
      integer("expert_mlp", &c->expert_mlp) && integer("self_attn_every_n_layers", &c->self_attn_every_n_layers) &&
      integer("n_lang", &c->n_lang) && integer("max_state_dim", &c->max_state_dim) &&
      integer("max_action_dim", &c->max_action_dim) && integer("action_dim", &c->action_dim) &&
      integer("chunk", &c->chunk) && integer("num_steps", &c->num_steps);
  if (!ok) return false;
  if (c->patch <= 0 || c->image_size % c->patch != 0 || c->scale_factor <= 0 || c->grid() % c->scale_factor != 0) {
    *err = "config: image_size must be a multiple of patch, and the patch grid of scale_factor";
    return false;
  }
  if (c->head_dim != 64 || c->vis_hidden != c->vis_heads * 64) {
    *err = "config: the attention kernels need head_dim 64 (vision and text)";
    return false;
  }
  if (c->n_cams < 1 || c->n_cams > 2) {
    *err = "config: the mask builder takes one or two cameras";
    return false;
  }
  if (c->kv_heads <= 0 || c->heads % c->kv_heads != 0) {
    *err = "config: heads must be a multiple of kv_heads";
    return false;
  }
  if (c->expert_layers != c->text_layers) {
    *err = "config: the expert must have one layer per text layer (each expert layer reads that layer's KV)";
    return false;
  }
  if (c->num_steps < 1 || c->chunk < 1 || c->n_lang < 1 || c->vis_layers < 1 || c->text_layers < 1) {
    *err = "config: empty dimension";
    return false;
  }
  return true;
}

// ----------------------------------------------------------------------------------------------- safetensors
struct TensorRec {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte offsets in the data section
  uint64_t arena_off = 0;       // offset in the device arena (256-byte aligned)
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
  }
};

int dtype_size(const std::string& d) {
  if (d == "I8" || d == "U8" || d == "BOOL") return 1;
  if (d == "BF16" || d == "F16" || d == "I16") return 2;
  if (d == "F32" || d == "I32") return 4;
  if (d == "F64" || d == "I64") return 8;
  return 0;
}

struct LinMeta {
  int n = 0, k = 0;
  std::string kind;  // "w8a8" | "w8a16" | "bf16"
  float act_scale = 1.0f;
};

struct PackedFile {
  Cfg cfg{};
  std::map<std::string, TensorRec> tensors;
  std::map<std::string, LinMeta> linears;
  uint64_t data_start = 0;  // file offset of the data section
  uint64_t arena_bytes = 0;
};

constexpr uint64_t kAlign = 256;
uint64_t align_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

struct File {
  FILE* f = nullptr;
  ~File() {
    if (f) std::fclose(f);
  }
};

// Reads and validates the header of a packed-weights file (no tensor data).
int32_t read_header(const char* path, PackedFile* pf, std::string* err) {
  if (!path) {
    *err = "null path";
    return SVLA_ERR_ARG;
  }
  File fh;
  fh.f = std::fopen(path, "rb");
  if (!fh.f) {
    *err = fmt("cannot open %s", path);
    return SVLA_ERR_ARG;
  }
  if (std::fseek(fh.f, 0, SEEK_END) != 0) {
    *err = "cannot seek";
    return SVLA_ERR_ARG;
  }
  const long long fsize = std::ftell(fh.f);
  std::fseek(fh.f, 0, SEEK_SET);
  unsigned char lenb[8];
  if (fsize < 8 || std::fread(lenb, 1, 8, fh.f) != 8) {
    *err = "file too short for a safetensors header";
    return SVLA_ERR_ARG;
  }
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | lenb[i];
  if (hlen == 0 || hlen > (100ull << 20) || hlen > static_cast<uint64_t>(fsize) - 8) {
    *err = fmt("bad safetensors header length %llu", static_cast<unsigned long long>(hlen));
    return SVLA_ERR_ARG;
  }
  std::string header(hlen, '\0');
  if (std::fread(&header[0], 1, hlen, fh.f) != hlen) {
    *err = "cannot read the safetensors header";
    return SVLA_ERR_ARG;
  }
  Json root;
  std::string jerr;
  if (!parse_json(header, &root, &jerr) || root.type != Json::kObj) {
    *err = "safetensors header: " + (jerr.empty() ? std::string("not an object") : jerr);
    return SVLA_ERR_ARG;
  }
  pf->data_start = 8 + hlen;
  const uint64_t data_bytes = static_cast<uint64_t>(fsize) - pf->data_start;
  const Json* meta = root.get("__metadata__");
  if (!meta || meta->type != Json::kObj) {
    *err = "no __metadata__: not a packed-weights file";
    return SVLA_ERR_ARG;
  }
  const Json* tag = meta->get("svla_packed");
  if (!tag || tag->type != Json::kStr || tag->str != "1") {
    *err = "metadata svla_packed != \"1\": not a packed-weights file";
    return SVLA_ERR_ARG;
  }
  const Json* cfg_s = meta->get("config");
  const Json* lin_s = meta->get("linears");
  if (!cfg_s || cfg_s->type != Json::kStr || !lin_s || lin_s->type != Json::kStr) {
    *err = "metadata lacks the config / linears JSON strings";
    return SVLA_ERR_ARG;
  }
  Json cfg_j, lin_j;
  if (!parse_json(cfg_s->str, &cfg_j, &jerr) || cfg_j.type != Json::kObj) {
    *err = "config metadata: " + jerr;
    return SVLA_ERR_ARG;
  }
  if (!read_cfg(cfg_j, &pf->cfg, err)) return SVLA_ERR_ARG;
  if (!parse_json(lin_s->str, &lin_j, &jerr) || lin_j.type != Json::kObj) {
    *err = "linears metadata: " + jerr;
    return SVLA_ERR_ARG;
  }
  for (const auto& kv : lin_j.obj) {
    const Json* n = kv.second.get("n");
    const Json* k = kv.second.get("k");
    const Json* kind = kv.second.get("kind");
    const Json* act = kv.second.get("act_scale");
    if (!n || !k || !kind || !act || n->type != Json::kNum || k->type != Json::kNum || kind->type != Json::kStr ||
        act->type != Json::kNum) {
      *err = "linears metadata: bad entry for " + kv.first;
      return SVLA_ERR_ARG;
    }
    if (kind->str != "w8a8" && kind->str != "w8a16" && kind->str != "bf16") {
      *err = "linears metadata: unknown kind " + kind->str + " for " + kv.first;
      return SVLA_ERR_ARG;
    }
    LinMeta m;
    m.n = static_cast<int>(n->num);
    m.k = static_cast<int>(k->num);
    m.kind = kind->str;
    m.act_scale = static_cast<float>(act->num);
    if (m.n <= 0 || m.k <= 0) {
      *err = "linears metadata: bad shape for " + kv.first;
      return SVLA_ERR_ARG;
    }
    pf->linears[kv.first] = m;
  }
  uint64_t off = 0;
  for (const auto& kv : root.obj) {
    if (kv.first == "__metadata__") continue;
    const Json& t = kv.second;
    const Json* dt = t.get("dtype");
    const Json* shape = t.get("shape");
    const Json* offs = t.get("data_offsets");
    if (!dt || dt->type != Json::kStr || !shape || shape->type != Json::kArr || !offs || offs->type != Json::kArr ||
        offs->arr.size() != 2) {
      *err = "bad tensor entry " + kv.first;
      return SVLA_ERR_ARG;
    }
    TensorRec r;
    r.dtype = dt->str;
    const int es = dtype_size(r.dtype);
    if (es == 0) {
      *err = "unsupported dtype " + r.dtype + " of " + kv.first;
      return SVLA_ERR_ARG;
    }
    for (const Json& s : shape->arr) {
      if (s.type != Json::kNum || s.num < 0) {
        *err = "bad shape of " + kv.first;
        return SVLA_ERR_ARG;
      }
      r.shape.push_back(static_cast<int64_t>(s.num));
    }
    r.begin = static_cast<uint64_t>(offs->arr[0].num);
    r.end = static_cast<uint64_t>(offs->arr[1].num);
    if (r.end < r.begin || r.end > data_bytes || r.end - r.begin != static_cast<uint64_t>(r.numel()) * es) {
      *err = "data offsets of " + kv.first + " do not match its shape or the file size";
      return SVLA_ERR_ARG;
    }
    r.arena_off = off;
    off = align_up(off + (r.end - r.begin), kAlign);
    pf->tensors[kv.first] = r;
  }
  pf->arena_bytes = off;
  return SVLA_OK;
}

// ----------------------------------------------------------------------------------------------- engine
struct Lin {
  int n = 0, k = 0;
  std::string kind;
  float act = 1.0f;
  const void* weight = nullptr;      // int8 [n, k] (w8a8 / w8a16) or bf16 [n, k] (bf16)
  const float* wscale = nullptr;     // fp32 [n]
  const void* bias = nullptr;        // bf16 [n]
  const float* smooth = nullptr;     // fp32 [k]
  const float* rsmooth = nullptr;    // fp32 [k]
  const void* weight_deq = nullptr;  // bf16 [n, k] (w8a16)
};

using Launch = std::function<int32_t(cudaStream_t)>;

struct PerBatch {
  std::vector<Launch> launches;
  cudaGraphExec_t exec = nullptr;
  int runs = 0;
};

// Device buffers of one call, sized for max_batch samples; the first B samples' rows serve a B-sample call
// (every buffer is batch-major).
struct Buffers {
  float* in_img;            // [B, n_cams, C, S, S]
  uint8_t* in_img_mask;     // [n_cams, B]
  int64_t* in_tokens;       // [B, n_lang]
  uint8_t* in_lang_mask;    // [B, n_lang]
  float* in_state;          // [B, max_state_dim]
  float* in_noise;          // [B, chunk, max_action_dim]
  void* state_bf;
  uint8_t *prefix_mask, *self_mask, *cross_mask;
  int32_t *prefix_pos, *suffix_pos, *cross_pos;
  void *patches, *vh;
  void* v_in[3];
  void* v_qkv[3];
  void *v_ctx, *v_fc1_in, *v_fc2_in, *conn_in;
  void* h;
  void* t_in[3];
  void* t_q;
  std::vector<void*> kcache, vcache, ck, cv;
  void *t_ctx, *t_mlp;
  void* t_mlp_in[2];
  float* xt;
  void *xt_bf, *a_emb, *a_t, *eh, *ey, *eq, *ek, *ev, *ectx, *emlp;
  // constants
  void* splitk_ws;
  size_t splitk_bytes;
  uint32_t* flow_sync;  // grid-barrier words of the persistent flow kernel
  float* flow_norm;     // its RMSNorm statistics scratch
  float* rope_cs;
  float* c_step;
};

}  // namespace engine_impl
}  // namespace svla

using namespace svla::engine_impl;
using svla::set_error;

struct svla_engine {
  Cfg cfg{};
  int max_batch = 0;
  int flags = 0;
  int device = 0;
  PackedFile file;
  char* weights = nullptr;  // device arena of the file's tensors
  char* arena = nullptr;    // device arena of the buffers
  char* flow_frag = nullptr;  // fragment-order copies of the weights the persistent flow kernel reads
  std::map<std::string, const void*> frag;  // linear -> its copy in flow_frag
  uint64_t arena_bytes = 0;
  Buffers buf{};
  std::map<std::string, Lin> lin;
  std::map<std::string, const void*> t;  // "t/<name>" tensors by name
  std::map<int, PerBatch> per_batch;
  cudaStream_t capture_stream = nullptr;
  int launches_per_call = 0;
};

namespace svla {
namespace engine_impl {

constexpr size_t kSplitKBytes = 32u << 20;  // split-K workspace shared by the call's GEMMs (stream-ordered)

int ld16(int n) { return (n + 15) / 16 * 16; }

float bf16_round(float x) {  // round to nearest even bfloat16, as a float
  uint32_t u;
  std::memcpy(&u, &x, 4);
  if ((u & 0x7F800000u) != 0x7F800000u) u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
  float r;
  std::memcpy(&r, &u, 4);
  return r;
}

const char* const kVision = "model.vlm_with_expert.vlm.model.vision_model";
const char* const kText = "model.vlm_with_expert.vlm.model.text_model";
const char* const kExpert = "model.vlm_with_expert.lm_expert";
const char* const kConnector = "model.vlm_with_expert.vlm.model.connector.modality_projection.proj";

// Checks that every tensor the call reads is present with the dtype and shape the config gives.
int32_t check_tensors(const PackedFile& pf, std::string* err) {
  const Cfg& c = pf.cfg;
  auto need = [&](const std::string& name, const char* dtype, std::vector<int64_t> shape) {
    auto it = pf.tensors.find(name);
    if (it == pf.tensors.end()) {
      *err = "packed file lacks " + name;
      return false;
    }
    if (it->second.dtype != dtype || it->second.shape != shape) {
      std::string s;
      for (int64_t d : it->second.shape) s += std::to_string(d) + ",";
      *err = fmt("%s: %s [%s] where %s was expected", name.c_str(), it->second.dtype.c_str(), s.c_str(), dtype);
      return false;
    }
    return true;
  };
  for (const auto& kv : pf.linears) {
    const LinMeta& m = kv.second;
    const std::string p = "lin/" + kv.first + "/";
    if (m.kind == "bf16") {
      if (!need(p + "weight", "BF16", {m.n, m.k})) return SVLA_ERR_ARG;
    } else {
      if (!need(p + "weight", "I8", {m.n, m.k}) || !need(p + "wscale", "F32", {m.n})) return SVLA_ERR_ARG;
    }
    if (m.kind == "w8a8" && (!need(p + "smooth", "F32", {m.k}) || !need(p + "rsmooth", "F32", {m.k})))
      return SVLA_ERR_ARG;
    if (m.kind == "w8a16" && !need(p + "weight_deq", "BF16", {m.n, m.k})) return SVLA_ERR_ARG;
    if (pf.tensors.count(p + "bias") && !need(p + "bias", "BF16", {m.n})) return SVLA_ERR_ARG;
  }
  auto lin = [&](const std::string& name, int n, int k, const char* kind) {
    auto it = pf.linears.find(name);
    if (it == pf.linears.end()) {
      *err = "packed file lacks the linear " + name;
      return false;
    }
    if (it->second.n != n || it->second.k != k) {
      *err = fmt("%s: [%d, %d] where [%d, %d] was expected", name.c_str(), it->second.n, it->second.k, n, k);
      return false;
    }
    if (kind && it->second.kind != kind) {
      *err = name + " must be " + kind + " (it feeds a fused quantiser), is " + it->second.kind;
      return false;
    }
    return true;
  };
  const int Hv = c.vis_hidden, H = c.hidden, E = c.expert_hidden;
  const std::string ve = std::string(kVision) + ".embeddings";
  if (!need("t/patch_w2d", "BF16", {Hv, c.channels * c.patch * c.patch}) ||
      !need("t/" + ve + ".patch_embedding.bias", "BF16", {Hv}) ||
      !need("t/" + ve + ".position_embedding.weight", "BF16", {c.n_patches(), Hv}) ||
      !need("t/" + std::string(kVision) + ".post_layernorm.weight", "BF16", {Hv}) ||
      !need("t/" + std::string(kVision) + ".post_layernorm.bias", "BF16", {Hv}) ||
      !need("t/" + std::string(kText) + ".embed_tokens.weight", "BF16", {c.vocab, H}) ||
      !need("t/" + std::string(kExpert) + ".norm.weight", "BF16", {E}) ||
      !need("t/time_embedding", "BF16", {c.num_steps, E}))
    return SVLA_ERR_ARG;
  for (int i = 0; i < c.vis_layers; ++i) {
    const std::string p = std::string(kVision) + ".encoder.layers." + std::to_string(i);
    for (const char* ln : {".layer_norm1", ".layer_norm2"})
      if (!need("t/" + p + ln + ".weight", "BF16", {Hv}) || !need("t/" + p + ln + ".bias", "BF16", {Hv}))
        return SVLA_ERR_ARG;
    for (const char* n : {".self_attn.q_proj", ".self_attn.k_proj", ".self_attn.v_proj", ".self_attn.out_proj"})
      if (!lin(p + n, Hv, Hv, "w8a8")) return SVLA_ERR_ARG;
    if (!lin(p + ".mlp.fc1", c.vis_mlp, Hv, "w8a8") || !lin(p + ".mlp.fc2", Hv, c.vis_mlp, "w8a8"))
      return SVLA_ERR_ARG;
  }
  if (!lin(kConnector, H, Hv * c.scale_factor * c.scale_factor, "w8a8")) return SVLA_ERR_ARG;
  for (int i = 0; i < c.text_layers; ++i) {
    const std::string p = std::string(kText) + ".layers." + std::to_string(i);
    if (!need("t/" + p + ".input_layernorm.weight", "BF16", {H}) ||
        !need("t/" + p + ".post_attention_layernorm.weight", "BF16", {H}))
      return SVLA_ERR_ARG;
    if (!lin(p + ".self_attn.q_proj", c.q_dim(), H, "w8a8") || !lin(p + ".self_attn.k_proj", c.kv_dim(), H, "w8a8") ||
        !lin(p + ".self_attn.v_proj", c.kv_dim(), H, "w8a8") || !lin(p + ".self_attn.o_proj", H, c.q_dim(), "w8a8") ||
        !lin(p + ".mlp.gate_proj", c.mlp, H, "w8a8") || !lin(p + ".mlp.up_proj", c.mlp, H, "w8a8") ||
        !lin(p + ".mlp.down_proj", H, c.mlp, nullptr))
      return SVLA_ERR_ARG;
  }
  for (int i = 0; i < c.expert_layers; ++i) {
    const std::string p = std::string(kExpert) + ".layers." + std::to_string(i);
    const int kv_in = c.is_cross(i) ? c.kv_dim() : E;
    if (!need("t/" + p + ".input_layernorm.weight", "BF16", {E}) ||
        !need("t/" + p + ".post_attention_layernorm.weight", "BF16", {E}))
      return SVLA_ERR_ARG;
    if (!lin(p + ".self_attn.q_proj", c.q_dim(), E, nullptr) ||
        !lin(p + ".self_attn.k_proj", c.kv_dim(), kv_in, nullptr) ||
        !lin(p + ".self_attn.v_proj", c.kv_dim(), kv_in, nullptr) ||
        !lin(p + ".self_attn.o_proj", E, c.q_dim(), nullptr) || !lin(p + ".mlp.gate_proj", c.expert_mlp, E, nullptr) ||
        !lin(p + ".mlp.up_proj", c.expert_mlp, E, nullptr) || !lin(p + ".mlp.down_proj", E, c.expert_mlp, nullptr))
      return SVLA_ERR_ARG;
  }
  if (!lin("model.state_proj", H, c.max_state_dim, "bf16") || !lin("model.action_in_proj", E, c.max_action_dim, "bf16") ||
      !lin("model.action_out_proj", c.max_action_dim, E, "bf16") ||
      !lin("model.action_time_mlp_in", E, 2 * E, "bf16") || !lin("model.action_time_mlp_out", E, E, "bf16"))
    return SVLA_ERR_ARG;
  for (const char* name : {"model.state_proj", "model.action_in_proj", "model.action_out_proj",
                           "model.action_time_mlp_in", "model.action_time_mlp_out"})
    if (!pf.tensors.count(std::string("lin/") + name + "/bias")) {
      *err = std::string(name) + " needs a bias";
      return SVLA_ERR_ARG;
    }
  return SVLA_OK;
}

void fill_info(const PackedFile& pf, svla_engine_info* info) {
  const Cfg& c = pf.cfg;
  std::memset(info, 0, sizeof(*info));
  info->n_cams = c.n_cams;
  info->channels = c.channels;
  info->image_size = c.image_size;
  info->n_lang = c.n_lang;
  info->max_state_dim = c.max_state_dim;
  info->max_action_dim = c.max_action_dim;
  info->chunk = c.chunk;
  info->num_steps = c.num_steps;
  info->action_dim = c.action_dim;
  info->prefix_len = c.prefix_len();
  info->vis_layers = c.vis_layers;
  info->text_layers = c.text_layers;
  info->expert_layers = c.expert_layers;
  info->n_linears = static_cast<int32_t>(pf.linears.size());
  info->n_tensors = static_cast<int32_t>(pf.tensors.size());
  info->weight_bytes = static_cast<int64_t>(pf.arena_bytes);
}

// Sub-allocates the call's buffers (256-byte aligned) from one arena; pass base = nullptr to size it.
uint64_t layout_buffers(const Cfg& c, int B, char* base, Buffers* b) {
  uint64_t off = 0;
  auto take = [&](uint64_t bytes) -> char* {
    char* p = base ? base + off : nullptr;
    off = align_up(off + bytes, kAlign);
    return p;
  };
  const uint64_t Lp = c.prefix_len(), S = c.chunk, NI = static_cast<uint64_t>(B) * c.n_cams;
  const uint64_t NV = NI * c.n_patches(), Hv = c.vis_hidden, H = c.hidden, E = c.expert_hidden;
  const uint64_t img = static_cast<uint64_t>(c.channels) * c.image_size * c.image_size;
  b->in_img = reinterpret_cast<float*>(take(NI * img * 4));
  b->in_img_mask = reinterpret_cast<uint8_t*>(take(NI));
  b->in_tokens = reinterpret_cast<int64_t*>(take(static_cast<uint64_t>(B) * c.n_lang * 8));
  b->in_lang_mask = reinterpret_cast<uint8_t*>(take(static_cast<uint64_t>(B) * c.n_lang));
  b->in_state = reinterpret_cast<float*>(take(static_cast<uint64_t>(B) * c.max_state_dim * 4));
  b->in_noise = reinterpret_cast<float*>(take(B * S * c.max_action_dim * 4));
  b->state_bf = take(static_cast<uint64_t>(B) * c.max_state_dim * 2);
  b->prefix_mask = reinterpret_cast<uint8_t*>(take(B * Lp * ld16(static_cast<int>(Lp))));
  b->self_mask = reinterpret_cast<uint8_t*>(take(B * S * ld16(static_cast<int>(Lp + S))));
  b->cross_mask = reinterpret_cast<uint8_t*>(take(B * S * ld16(static_cast<int>(Lp))));
  b->prefix_pos = reinterpret_cast<int32_t*>(take(B * Lp * 4));
  b->suffix_pos = reinterpret_cast<int32_t*>(take(B * S * 4));
  b->cross_pos = reinterpret_cast<int32_t*>(take(B * S * 4));
  b->patches = take(NV * c.channels * c.patch * c.patch * 2);
  b->vh = take(NV * Hv * 2);
  for (auto& p : b->v_in) p = take(NV * Hv);
  for (auto& p : b->v_qkv) p = take(NV * Hv * 2);
  b->v_ctx = take(NV * Hv);
  b->v_fc1_in = take(NV * Hv);
  b->v_fc2_in = take(NV * c.vis_mlp);
  b->conn_in = take(NI * c.n_img_tokens() * Hv * c.scale_factor * c.scale_factor);
  b->h = take(B * Lp * H * 2);
  for (auto& p : b->t_in) p = take(B * Lp * H);
  b->t_q = take(B * Lp * c.q_dim() * 2);
  b->kcache.assign(c.text_layers, nullptr);
  b->vcache.assign(c.text_layers, nullptr);
  for (int i = 0; i < c.text_layers; ++i) {
    b->kcache[i] = take(B * Lp * c.kv_dim() * 2);
    b->vcache[i] = take(B * Lp * c.kv_dim() * 2);
  }
  b->t_ctx = take(B * Lp * c.q_dim());
  for (auto& p : b->t_mlp_in) p = take(B * Lp * H);
  b->t_mlp = take(B * Lp * c.mlp * 2);
  b->ck.assign(c.expert_layers, nullptr);
  b->cv.assign(c.expert_layers, nullptr);
  for (int i = 0; i < c.expert_layers; ++i) {
    if (!c.is_cross(i)) continue;
    b->ck[i] = take(B * Lp * c.kv_dim() * 2);
    b->cv[i] = take(B * Lp * c.kv_dim() * 2);
  }
  b->xt = reinterpret_cast<float*>(take(B * S * c.max_action_dim * 4));
  b->xt_bf = take(B * S * c.max_action_dim * 2);
  b->a_emb = take(B * S * E * 2);
  b->a_t = take(B * S * E * 2);
  b->eh = take(B * S * E * 2);
  b->ey = take(B * S * E * 2);
  b->eq = take(B * S * c.q_dim() * 2);
  b->ek = take(B * S * c.kv_dim() * 2);
  b->ev = take(B * S * c.kv_dim() * 2);
  b->ectx = take(B * S * c.q_dim() * 2);
  b->emlp = take(B * S * c.expert_mlp * 2);
  b->splitk_bytes = kSplitKBytes;
  b->splitk_ws = take(kSplitKBytes);
  b->flow_sync = reinterpret_cast<uint32_t*>(take(8));
  b->flow_norm = reinterpret_cast<float*>(take(64 * 64 * 4));
  const int max_pos = c.prefix_len() + c.chunk;
  b->rope_cs = reinterpret_cast<float*>(take(static_cast<uint64_t>(max_pos) * 32 * 2 * 4));
  b->c_step = reinterpret_cast<float*>(take(static_cast<uint64_t>(c.num_steps) * E * 4));
  return off;
}

// ------------------------------------------------------------------ launch-list builder
// One sample_actions call for B samples (the order and descriptors of SmolVLARunner._build, quant mode).
class Builder {
 public:
  Builder(const svla_engine& e, int B, std::vector<Launch>* out) : e_(e), c_(e.cfg), b_(e.buf), B_(B), out_(out) {}

  void build() {
    const Cfg& c = c_;
    const Buffers& b = b_;
    const int B = B_;
    const int Lp = c.prefix_len(), S = c.chunk, H = c.hidden, E = c.expert_hidden, Hv = c.vis_hidden;
    const int NI = B * c.n_cams, NV = NI * c.n_patches();
    const int max_pos = Lp + S;
    // masks and positions
    {
      const uint8_t* m0 = b.in_img_mask;
      const uint8_t* m1 = c.n_cams > 1 ? b.in_img_mask + B : b.in_img_mask;
      const uint8_t* lm = b.in_lang_mask;
      uint8_t *pm = b.prefix_mask, *sm = b.self_mask, *cm = b.cross_mask;
      int32_t *pp = b.prefix_pos, *sp = b.suffix_pos, *cp = b.cross_pos;
      const int n_img = c.n_img_tokens(), n_lang = c.n_lang;
      add([=](cudaStream_t s) {
        return svla_build_masks(m0, m1, lm, B, n_img, n_lang, S, pm, pp, sm, cm, sp, cp, st(s));
      });
    }
    // ---------------- vision tower
    {
      const int C = c.channels, SZ = c.image_size, P = c.patch;
      const float* img = b.in_img;
      void* patches = b.patches;
      add([=](cudaStream_t s) { return svla_im2col(img, NI, C, SZ, P, patches, st(s)); });
    }
    const std::string ve = std::string(kVision) + ".embeddings";
    const int cpp = c.channels * c.patch * c.patch;
    {
      svla_gemm_desc d = desc(SVLA_KIND_BF16, SVLA_EPI_RESID, NV, cpp);
      d.nseg = 1;
      d.seg[0] = raw_seg(b.patches, cpp, tensor("patch_w2d"), cpp, b.vh, Hv, Hv);
      d.seg[0].bias = tensor(ve + ".patch_embedding.bias");
      d.resid = tensor(ve + ".position_embedding.weight");
      d.ldr = Hv;
      d.resid_rows = c.n_patches();
      gemm(d);
    }
    for (int i = 0; i < c.vis_layers; ++i) {
      const std::string p = std::string(kVision) + ".encoder.layers." + std::to_string(i);
      const std::string q = p + ".self_attn.q_proj", k = p + ".self_attn.k_proj", v = p + ".self_attn.v_proj";
      const std::string o = p + ".self_attn.out_proj", fc1 = p + ".mlp.fc1", fc2 = p + ".mlp.fc2";
      norm_quant(b.vh, Hv, NV, Hv, tensor("t/" + p + ".layer_norm1.weight"), c.vis_eps,
                 tensor("t/" + p + ".layer_norm1.bias"), {q, k, v}, {b.v_in[0], b.v_in[1], b.v_in[2]}, Hv);
      {
        svla_gemm_desc d = desc(kind(q, NV), SVLA_EPI_BF16, NV, Hv);
        d.nseg = 3;
        d.seg[0] = lin_seg(q, b.v_in[0], Hv, NV, b.v_qkv[0], Hv);
        d.seg[1] = lin_seg(k, b.v_in[1], Hv, NV, b.v_qkv[1], Hv);
        d.seg[2] = lin_seg(v, b.v_in[2], Hv, NV, b.v_qkv[2], Hv);
        gemm(d);
      }
      {
        svla_attn_desc a = attn(b.v_qkv[0], Hv, b.v_qkv[1], b.v_qkv[2], Hv, c.n_patches(), NI, c.n_patches(),
                                c.vis_heads, c.vis_heads);
        quant_out(&a, o, b.v_ctx, Hv, c.n_patches());
        attention(a);
      }
      resid_gemm(o, b.v_ctx, Hv, NV, b.vh, Hv);
      norm_quant(b.vh, Hv, NV, Hv, tensor("t/" + p + ".layer_norm2.weight"), c.vis_eps,
                 tensor("t/" + p + ".layer_norm2.bias"), {fc1}, {b.v_fc1_in}, Hv);
      {
        const Lin& f2 = e_.lin.at(fc2);
        svla_gemm_desc d = desc(SVLA_KIND_I8, SVLA_EPI_GELU_QUANT, NV, Hv);
        d.nseg = 1;
        d.seg[0] = lin_seg(fc1, b.v_fc1_in, Hv, NV, nullptr, 0);
        d.q_smooth = f2.smooth;
        d.q_rsmooth = f2.rsmooth;
        d.q_act = f2.act;
        d.qout = static_cast<int8_t*>(b.v_fc2_in);
        d.ldq = c.vis_mlp;
        gemm(d);
      }
      resid_gemm(fc2, b.v_fc2_in, c.vis_mlp, NV, b.vh, Hv);
    }
    // post LayerNorm + pixel shuffle + connector quantisation
    const int sf2 = c.scale_factor * c.scale_factor;
    {
      svla_norm_desc d = norm_desc(b.vh, Hv, NV, Hv, tensor("t/" + std::string(kVision) + ".post_layernorm.weight"),
                                   c.vis_eps, tensor("t/" + std::string(kVision) + ".post_layernorm.bias"));
      quant_outs(&d, {kConnector}, {b.conn_in}, Hv * sf2);
      d.pixel_shuffle = c.scale_factor;
      d.ps_grid = c.grid();
      norm(d);
    }
    // connector -> prefix rows (b, cam, token) -> b*Lp + cam*n_img + token, x bf16(sqrt(H)) in bf16
    {
      const int m = NI * c.n_img_tokens();
      svla_gemm_desc d = desc(kind(kConnector, m), SVLA_EPI_BF16, m, Hv * sf2);
      d.nseg = 1;
      d.seg[0] = lin_seg(kConnector, b.conn_in, Hv * sf2, m, b.h, H);
      d.post_scale = bf16_round(static_cast<float>(std::sqrt(static_cast<double>(H))));
      d.rows_per_group = c.n_cams * c.n_img_tokens();
      d.group_stride = Lp;
      gemm(d);
    }
    // language tokens x sqrt(H) and the state token
    {
      const void* table = tensor("t/" + std::string(kText) + ".embed_tokens.weight");
      const int n_lang = c.n_lang, vocab = c.vocab, row0 = c.n_cams * c.n_img_tokens();
      const float scale = static_cast<float>(std::sqrt(static_cast<double>(H)));
      const int64_t* tokens = b.in_tokens;
      void* h = b.h;
      add([=](cudaStream_t s) {
        return svla_embed_tokens(tokens, B, n_lang, table, vocab, H, scale, h, Lp, row0, st(s));
      });
      const int64_t n = static_cast<int64_t>(B) * c.max_state_dim;
      const float* state = b.in_state;
      void* state_bf = b.state_bf;
      add([=](cudaStream_t s) { return svla_f32_to_bf16(state, state_bf, n, st(s)); });
      svla_gemm_desc d = desc(SVLA_KIND_BF16, SVLA_EPI_BF16, B, c.max_state_dim);
      d.nseg = 1;
      d.seg[0] = lin_seg("model.state_proj", b.state_bf, c.max_state_dim, B, b.h, H);
      d.rows_per_group = 1;
      d.group_stride = Lp;
      d.row_offset = Lp - 1;
      gemm(d);
    }
    // ---------------- text layers (KV fill); the last layer's o_proj and MLP feed nothing sample_actions returns
    const int M = B * Lp;
    for (int i = 0; i < c.text_layers; ++i) {
      const std::string p = std::string(kText) + ".layers." + std::to_string(i);
      const std::string q = p + ".self_attn.q_proj", k = p + ".self_attn.k_proj", v = p + ".self_attn.v_proj";
      norm_quant(b.h, H, M, H, tensor("t/" + p + ".input_layernorm.weight"), c.rms_eps, nullptr, {q, k, v},
                 {b.t_in[0], b.t_in[1], b.t_in[2]}, H);
      {
        svla_gemm_desc d = desc(kind(q, M), SVLA_EPI_ROPE, M, H);
        d.nseg = 3;
        d.seg[0] = lin_seg(q, b.t_in[0], H, M, b.t_q, c.q_dim(), 1);
        d.seg[1] = lin_seg(k, b.t_in[1], H, M, b.kcache[i], c.kv_dim(), 1);
        d.seg[2] = lin_seg(v, b.t_in[2], H, M, b.vcache[i], c.kv_dim(), 0);
        rope(&d, b.prefix_pos, max_pos);
        gemm(d);
      }
      if (i == c.text_layers - 1) break;
      {
        svla_attn_desc a = attn(b.t_q, c.q_dim(), b.kcache[i], b.vcache[i], c.kv_dim(), Lp, B, Lp, c.heads, c.kv_heads);
        a.mask = b.prefix_mask;
        a.mask_bs = static_cast<int64_t>(Lp) * ld16(Lp);
        a.mask_rs = ld16(Lp);
        quant_out(&a, p + ".self_attn.o_proj", b.t_ctx, c.q_dim(), Lp);
        attention(a);
      }
      resid_gemm(p + ".self_attn.o_proj", b.t_ctx, c.q_dim(), M, b.h, H);
      const std::string g = p + ".mlp.gate_proj", u = p + ".mlp.up_proj";
      norm_quant(b.h, H, M, H, tensor("t/" + p + ".post_attention_layernorm.weight"), c.rms_eps, nullptr, {g, u},
                 {b.t_mlp_in[0], b.t_mlp_in[1]}, H);
      {
        svla_gemm_desc d = desc(kind(g, M), SVLA_EPI_SILU_MUL, M, H);
        d.nseg = 2;
        d.pair = 1;
        d.seg[0] = lin_seg(g, b.t_mlp_in[0], H, M, b.t_mlp, c.mlp);
        d.seg[1] = lin_seg(u, b.t_mlp_in[1], H, M, b.t_mlp, c.mlp);
        gemm(d);
      }
      resid_gemm(p + ".mlp.down_proj", b.t_mlp, c.mlp, M, b.h, H);
    }
    // ---------------- cross-attention K/V of the cached prefix (step-invariant)
    for (int i = 0; i < c.expert_layers; ++i) {
      if (!c.is_cross(i)) continue;
      const std::string p = std::string(kExpert) + ".layers." + std::to_string(i) + ".self_attn";
      svla_gemm_desc d = desc(kind(p + ".k_proj", M), SVLA_EPI_BF16, M, c.kv_dim());
      d.nseg = 2;
      d.seg[0] = lin_seg(p + ".k_proj", b.kcache[i], c.kv_dim(), M, b.ck[i], c.kv_dim());
      d.seg[1] = lin_seg(p + ".v_proj", b.vcache[i], c.kv_dim(), M, b.cv[i], c.kv_dim());
      gemm(d);
    }
    // ---------------- flow matching
    const int MS = B * S, A = c.max_action_dim;
    if (use_flow()) {
      flow(MS);
      return;
    }
    {
      const int64_t n = static_cast<int64_t>(MS) * A;
      const float* noise = b.in_noise;
      float* xt = b.xt;
      void* xt_bf = b.xt_bf;
      add([=](cudaStream_t s) { return svla_euler_init(noise, xt, xt_bf, n, st(s)); });
    }
    const float dt = static_cast<float>(-1.0 / c.num_steps);
    const Lin& mi = e_.lin.at("model.action_time_mlp_in");
    const std::string ep = kExpert;
    for (int step = 0; step < c.num_steps; ++step) {
      {
        svla_gemm_desc d = desc(SVLA_KIND_BF16, SVLA_EPI_BF16, MS, A);
        d.nseg = 1;
        d.seg[0] = lin_seg("model.action_in_proj", b.xt_bf, A, MS, b.a_emb, E);
        gemm(d);
      }
      {
        // time MLP in: W[:, :E] . action_emb + (W[:, E:] . time_emb(t_step) + b), the second term a constant
        svla_gemm_desc d = desc(SVLA_KIND_BF16, SVLA_EPI_SILU, MS, E);
        d.nseg = 1;
        d.seg[0] = raw_seg(b.a_emb, E, mi.weight, 2 * E, b.a_t, E, E);
        d.seg[0].bias_f32 = b.c_step + static_cast<size_t>(step) * E;
        gemm(d);
      }
      {
        svla_gemm_desc d = desc(SVLA_KIND_BF16, SVLA_EPI_BF16, MS, E);
        d.nseg = 1;
        d.seg[0] = lin_seg("model.action_time_mlp_out", b.a_t, E, MS, b.eh, E);
        gemm(d);
      }
      for (int i = 0; i < c.expert_layers; ++i) {
        const std::string p = ep + ".layers." + std::to_string(i);
        const std::string q = p + ".self_attn.q_proj";
        norm_y(b.eh, E, MS, E, tensor("t/" + p + ".input_layernorm.weight"), c.rms_eps, b.ey);
        if (c.is_cross(i)) {
          svla_gemm_desc d = desc(kind(q, MS), SVLA_EPI_ROPE, MS, E);
          d.nseg = 1;
          d.seg[0] = lin_seg(q, b.ey, E, MS, b.eq, c.q_dim(), 1);
          rope(&d, b.cross_pos, max_pos);
          gemm(d);
          svla_attn_desc a = attn(b.eq, c.q_dim(), b.ck[i], b.cv[i], c.kv_dim(), Lp, B, S, c.heads, c.kv_heads);
          key_pad(&a, Lp, S);
          bf16_out(&a, b.ectx, c.q_dim(), S);
          attention(a);
        } else {
          svla_gemm_desc d = desc(kind(q, MS), SVLA_EPI_ROPE, MS, E);
          d.nseg = 3;
          d.seg[0] = lin_seg(q, b.ey, E, MS, b.eq, c.q_dim(), 1);
          d.seg[1] = lin_seg(p + ".self_attn.k_proj", b.ey, E, MS, b.ek, c.kv_dim(), 1);
          d.seg[2] = lin_seg(p + ".self_attn.v_proj", b.ey, E, MS, b.ev, c.kv_dim(), 0);
          rope(&d, b.suffix_pos, max_pos);
          gemm(d);
          svla_attn_desc a =
              attn(b.eq, c.q_dim(), b.kcache[i], b.vcache[i], c.kv_dim(), Lp, B, S, c.heads, c.kv_heads);
          a.k2 = b.ek;
          a.v2 = b.ev;
          a.kv2_bs = static_cast<int64_t>(S) * c.kv_dim();
          a.kv2_rs = c.kv_dim();
          a.l2 = S;
          key_pad(&a, Lp, S);
          bf16_out(&a, b.ectx, c.q_dim(), S);
          attention(a);
        }
        resid_gemm(p + ".self_attn.o_proj", b.ectx, c.q_dim(), MS, b.eh, E);
        norm_y(b.eh, E, MS, E, tensor("t/" + p + ".post_attention_layernorm.weight"), c.rms_eps, b.ey);
        {
          const std::string g = p + ".mlp.gate_proj";
          svla_gemm_desc d = desc(kind(g, MS), SVLA_EPI_SILU_MUL, MS, E);
          d.nseg = 2;
          d.pair = 1;
          d.seg[0] = lin_seg(g, b.ey, E, MS, b.emlp, c.expert_mlp);
          d.seg[1] = lin_seg(p + ".mlp.up_proj", b.ey, E, MS, b.emlp, c.expert_mlp);
          gemm(d);
        }
        resid_gemm(p + ".mlp.down_proj", b.emlp, c.expert_mlp, MS, b.eh, E);
      }
      norm_y(b.eh, E, MS, E, tensor("t/" + ep + ".norm.weight"), c.rms_eps, b.ey);
      {
        svla_gemm_desc d = desc(SVLA_KIND_BF16, SVLA_EPI_EULER, MS, E);
        d.nseg = 1;
        d.seg[0] = lin_seg("model.action_out_proj", b.ey, E, MS, nullptr, 0);
        d.dt = dt;
        d.xt = b.xt;
        d.xt_bf16 = b.xt_bf;
        gemm(d);
      }
    }
  }

 private:
  const svla_engine& e_;
  const Cfg& c_;
  const Buffers& b_;
  const int B_;
  std::vector<Launch>* out_;

  static svla_stream_t st(cudaStream_t s) { return reinterpret_cast<svla_stream_t>(s); }

  // the persistent flow kernel applies: few action rows and its weights packed (flow_weights_packed)
  bool use_flow() const { return !e_.frag.empty() && B_ * c_.chunk <= SVLA_FLOW_MAX_ROWS; }

  const void* frag(const std::string& name) const { return e_.frag.at(name); }
  const float* wscale(const std::string& name) const { return e_.lin.at(name).wscale; }

  void flow(int MS) {
    const Cfg& c = c_;
    const Buffers& b = b_;
    svla_flow_desc d;
    std::memset(&d, 0, sizeof(d));
    d.batch = B_;
    d.chunk = c.chunk;
    d.prefix_len = c.prefix_len();
    d.hidden = c.expert_hidden;
    d.action_dim = c.max_action_dim;
    d.heads = c.heads;
    d.kv_heads = c.kv_heads;
    d.mlp = c.expert_mlp;
    d.n_layers = c.expert_layers;
    d.num_steps = c.num_steps;
    d.eps = static_cast<float>(c.rms_eps);
    d.noise = b.in_noise;
    d.xt = b.xt;
    d.xt_bf16 = b.xt_bf;
    d.w_action_in = frag("model.action_in_proj");
    d.b_action_in = e_.lin.at("model.action_in_proj").bias;
    d.w_time_in = frag("model.action_time_mlp_in");
    d.time_in_const = b.c_step;
    d.w_time_out = frag("model.action_time_mlp_out");
    d.b_time_out = e_.lin.at("model.action_time_mlp_out").bias;
    d.final_norm = tensor(std::string(kExpert) + ".norm.weight");
    d.w_action_out = frag("model.action_out_proj");
    d.b_action_out = e_.lin.at("model.action_out_proj").bias;
    d.key_mask = b.cross_mask;
    d.key_mask_bs = static_cast<int64_t>(c.chunk) * ld16(c.prefix_len());
    d.suffix_pos = b.suffix_pos;
    d.cross_pos = b.cross_pos;
    d.rope_cs = b.rope_cs;
    d.max_pos = c.prefix_len() + c.chunk;
    d.a_emb = b.a_emb;
    d.a_t = b.a_t;
    d.eh = b.eh;
    d.eq = b.eq;
    d.ek = b.ek;
    d.ev = b.ev;
    d.ectx = b.ectx;
    d.emlp = b.emlp;
    d.norm_part = b.flow_norm;
    d.sync = b.flow_sync;
    for (int i = 0; i < c.expert_layers; ++i) {
      const std::string p = std::string(kExpert) + ".layers." + std::to_string(i);
      svla_flow_layer& l = d.layer[i];
      l.input_norm = tensor(p + ".input_layernorm.weight");
      l.post_norm = tensor(p + ".post_attention_layernorm.weight");
      l.wq = frag(p + ".self_attn.q_proj");
      l.sq = wscale(p + ".self_attn.q_proj");
      l.wo = frag(p + ".self_attn.o_proj");
      l.so = wscale(p + ".self_attn.o_proj");
      l.wg = frag(p + ".mlp.gate_proj");
      l.sg = wscale(p + ".mlp.gate_proj");
      l.wu = frag(p + ".mlp.up_proj");
      l.su = wscale(p + ".mlp.up_proj");
      l.wd = frag(p + ".mlp.down_proj");
      l.sd = wscale(p + ".mlp.down_proj");
      l.cross = c.is_cross(i) ? 1 : 0;
      if (l.cross) {
        l.keys = b.ck[i];
        l.values = b.cv[i];
      } else {
        l.wk = frag(p + ".self_attn.k_proj");
        l.sk = wscale(p + ".self_attn.k_proj");
        l.wv = frag(p + ".self_attn.v_proj");
        l.sv = wscale(p + ".self_attn.v_proj");
        l.keys = b.kcache[i];
        l.values = b.vcache[i];
      }
    }
    (void)MS;
    add([d](cudaStream_t s) { return svla_flow(&d, st(s)); });
  }
  void add(Launch f) { out_->push_back(std::move(f)); }

  const void* tensor(const std::string& name) const {
    const std::string key = name.compare(0, 2, "t/") == 0 ? name : "t/" + name;
    auto it = e_.t.find(key);
    return it == e_.t.end() ? nullptr : it->second;  // presence checked when the file was loaded
  }

  svla_gemm_desc desc(int kind, int epi, int m, int k) const {
    svla_gemm_desc d;
    std::memset(&d, 0, sizeof(d));
    d.kind = kind;
    d.epi = epi;
    d.m = m;
    d.k = k;
    // every B operand is a packed weight written at load time
    d.weights_resident = 1;
    if (!(e_.flags & SVLA_ENGINE_NO_SPLIT_K)) {
      d.workspace = b_.splitk_ws;
      d.workspace_bytes = b_.splitk_bytes;
    }
    return d;
  }

  static svla_gemm_seg raw_seg(const void* a, int lda, const void* w, int ldb, void* out, int ldo, int n) {
    svla_gemm_seg s;
    std::memset(&s, 0, sizeof(s));
    s.a = a;
    s.lda = lda;
    s.b = w;
    s.ldb = ldb;
    s.out = out;
    s.ldo = out ? ldo : n;
    s.n = n;
    s.act_scale = 1.0f;
    return s;
  }

  // W8A16 linears multiply by the stored bf16(q * wscale) weight (a bf16 GEMM) at every row count
  static bool deq_rows(const Lin& p, int m) { return p.kind == "w8a16" && m >= 1; }

  int kind(const std::string& name, int m) const {
    const Lin& p = e_.lin.at(name);
    if (p.kind == "bf16" || deq_rows(p, m)) return SVLA_KIND_BF16;
    return p.kind == "w8a8" ? SVLA_KIND_I8 : SVLA_KIND_W8A16;
  }

  svla_gemm_seg lin_seg(const std::string& name, const void* a, int lda, int m, void* out, int ldo,
                        int rope = 0) const {
    const Lin& p = e_.lin.at(name);
    svla_gemm_seg s = raw_seg(a, lda, p.weight, p.k, out, ldo, p.n);
    s.bias = p.bias;
    s.rope = rope;
    if (p.kind == "bf16") return s;
    if (deq_rows(p, m)) {
      s.b = p.weight_deq;
      return s;
    }
    s.wscale = p.wscale;
    if (p.kind == "w8a8") s.act_scale = p.act;
    return s;
  }

  void gemm(const svla_gemm_desc& d) {
    add([d](cudaStream_t s) { return svla_gemm(&d, st(s)); });
  }

  void resid_gemm(const std::string& name, const void* a, int k, int m, void* out, int ld) {
    svla_gemm_desc d = desc(kind(name, m), SVLA_EPI_RESID, m, k);
    d.nseg = 1;
    d.seg[0] = lin_seg(name, a, k, m, out, ld);
    d.resid = out;
    d.ldr = ld;
    gemm(d);
  }

  void rope(svla_gemm_desc* d, const int32_t* pos, int max_pos) const {
    d->rope_cs = b_.rope_cs;
    d->pos = pos;
    d->max_pos = max_pos;
  }

  svla_norm_desc norm_desc(const void* x, int ldx, int m, int k, const void* w, double eps, const void* bias) const {
    svla_norm_desc d;
    std::memset(&d, 0, sizeof(d));
    d.x = x;
    d.ldx = ldx;
    d.weight = w;
    d.bias = bias;
    d.eps = static_cast<float>(eps);
    d.layernorm = bias ? 1 : 0;
    d.m = m;
    d.k = k;
    return d;
  }

  void quant_outs(svla_norm_desc* d, const std::vector<std::string>& mods, const std::vector<void*>& outs,
                  int ldq) const {
    for (size_t i = 0; i < mods.size(); ++i) {
      const Lin& p = e_.lin.at(mods[i]);
      d->q[i] = static_cast<int8_t*>(outs[i]);
      d->smooth[i] = p.smooth;
      d->rsmooth[i] = p.rsmooth;
      d->act[i] = p.act;
    }
    d->nq = static_cast<int32_t>(mods.size());
    d->ldq = ldq;
  }

  void norm(const svla_norm_desc& d) {
    add([d](cudaStream_t s) { return svla_norm_quant(&d, st(s)); });
  }

  void norm_quant(const void* x, int ldx, int m, int k, const void* w, double eps, const void* bias,
                  const std::vector<std::string>& mods, const std::vector<void*>& outs, int ldq) {
    svla_norm_desc d = norm_desc(x, ldx, m, k, w, eps, bias);
    quant_outs(&d, mods, outs, ldq);
    norm(d);
  }

  void norm_y(const void* x, int ldx, int m, int k, const void* w, double eps, void* y) {
    svla_norm_desc d = norm_desc(x, ldx, m, k, w, eps, nullptr);
    d.y = y;
    d.ldy = k;
    norm(d);
  }

  // attention over `batch` sequences of lq queries; k/v [batch, l1, kv_cols]
  static svla_attn_desc attn(const void* q, int q_cols, const void* k1, const void* v1, int kv_cols, int l1,
                             int batch, int lq, int hq, int hkv) {
    svla_attn_desc a;
    std::memset(&a, 0, sizeof(a));
    a.q = q;
    a.q_bs = static_cast<int64_t>(lq) * q_cols;
    a.q_rs = q_cols;
    a.k1 = k1;
    a.v1 = v1;
    a.kv1_bs = static_cast<int64_t>(l1) * kv_cols;
    a.kv1_rs = kv_cols;
    a.l1 = l1;
    a.batch = batch;
    a.lq = lq;
    a.hq = hq;
    a.hkv = hkv;
    a.impl = SVLA_ATTN_AUTO;
    return a;
  }

  void quant_out(svla_attn_desc* a, const std::string& mod, void* qo, int cols, int lq) const {
    const Lin& p = e_.lin.at(mod);
    a->qo = static_cast<int8_t*>(qo);
    a->qo_bs = static_cast<int64_t>(lq) * cols;
    a->qo_rs = cols;
    a->qo_smooth = p.smooth;
    a->qo_rsmooth = p.rsmooth;
    a->qo_act = p.act;
  }

  static void bf16_out(svla_attn_desc* a, void* o, int cols, int lq) {
    a->o = o;
    a->o_bs = static_cast<int64_t>(lq) * cols;
    a->o_rs = cols;
  }

  // the prefix key padding (row 0 of the cross mask of each sample), causal order over the chunk
  void key_pad(svla_attn_desc* a, int Lp, int S) const {
    a->key_mask = b_.cross_mask;
    a->key_mask_bs = static_cast<int64_t>(S) * ld16(Lp);
    a->mask_keys = Lp;
  }

  void attention(const svla_attn_desc& a) {
    add([a](cudaStream_t s) { return svla_attention(&a, st(s)); });
  }
};

int32_t cuda_fail(cudaError_t e, const char* what) {
  return set_error(SVLA_ERR_CUDA, fmt("%s: %s", what, cudaGetErrorString(e)));
}

int32_t run_list(const std::vector<Launch>& list, cudaStream_t s) {
  for (const Launch& f : list) {
    const int32_t rc = f(s);
    if (rc != SVLA_OK) return rc;  // the failing entry point set the message
  }
  return SVLA_OK;
}

int32_t load_weights(svla_engine* e, const char* path, cudaStream_t stream) {
  const PackedFile& pf = e->file;
  std::vector<char> host(pf.arena_bytes, 0);
  File fh;
  fh.f = std::fopen(path, "rb");
  if (!fh.f) return set_error(SVLA_ERR_ARG, fmt("cannot open %s", path));
  for (const auto& kv : pf.tensors) {
    const TensorRec& r = kv.second;
    const uint64_t n = r.end - r.begin;
    if (n == 0) continue;
    if (std::fseek(fh.f, static_cast<long>(pf.data_start + r.begin), SEEK_SET) != 0 ||
        std::fread(host.data() + r.arena_off, 1, n, fh.f) != n)
      return set_error(SVLA_ERR_ARG, "cannot read the data of " + kv.first);
  }
  cudaError_t err = cudaMalloc(&e->weights, pf.arena_bytes ? pf.arena_bytes : kAlign);
  if (err != cudaSuccess) {
    e->weights = nullptr;
    return cuda_fail(err, "cudaMalloc(weights)");
  }
  err = cudaMemcpyAsync(e->weights, host.data(), pf.arena_bytes, cudaMemcpyHostToDevice, stream);
  if (err == cudaSuccess) err = cudaStreamSynchronize(stream);  // `host` is released on return
  if (err != cudaSuccess) return cuda_fail(err, "uploading the weights");
  auto ptr = [&](const std::string& name) -> void* {
    auto it = pf.tensors.find(name);
    return it == pf.tensors.end() ? nullptr : e->weights + it->second.arena_off;
  };
  for (const auto& kv : pf.linears) {
    Lin l;
    l.n = kv.second.n;
    l.k = kv.second.k;
    l.kind = kv.second.kind;
    l.act = kv.second.act_scale;
    const std::string p = "lin/" + kv.first + "/";
    l.weight = ptr(p + "weight");
    l.wscale = static_cast<const float*>(ptr(p + "wscale"));
    l.bias = ptr(p + "bias");
    l.smooth = static_cast<const float*>(ptr(p + "smooth"));
    l.rsmooth = static_cast<const float*>(ptr(p + "rsmooth"));
    l.weight_deq = ptr(p + "weight_deq");
    e->lin[kv.first] = l;
  }
  for (const auto& kv : pf.tensors)
    if (kv.first.compare(0, 2, "t/") == 0) e->t[kv.first] = e->weights + kv.second.arena_off;
  return SVLA_OK;
}

// rope table and the per-step constant of action_time_mlp_in: W[:, E:] . bf16(time_emb(t_k)) + b (fp32)
int32_t compute_constants(svla_engine* e, cudaStream_t stream) {
  const Cfg& c = e->cfg;
  const int E = c.expert_hidden;
  int32_t rc = svla_rope_table(e->buf.rope_cs, c.prefix_len() + c.chunk, static_cast<float>(c.rope_wavelength),
                               reinterpret_cast<svla_stream_t>(stream));
  if (rc != SVLA_OK) return rc;
  const Lin& mi = e->lin.at("model.action_time_mlp_in");
  svla_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.kind = SVLA_KIND_BF16;
  d.epi = SVLA_EPI_F32;
  d.m = c.num_steps;
  d.k = E;
  d.nseg = 1;
  svla_gemm_seg& s = d.seg[0];
  s.a = e->t.at("t/time_embedding");
  s.lda = E;
  s.b = static_cast<const char*>(mi.weight) + static_cast<size_t>(E) * 2;  // columns E.. of [E, 2E]
  s.ldb = 2 * E;
  s.bias = mi.bias;
  s.out = e->buf.c_step;
  s.ldo = E;
  s.n = E;
  s.act_scale = 1.0f;
  rc = svla_gemm(&d, reinterpret_cast<svla_stream_t>(stream));
  if (rc != SVLA_OK) return rc;
  const cudaError_t err = cudaStreamSynchronize(stream);
  return err == cudaSuccess ? SVLA_OK : cuda_fail(err, "computing the engine constants");
}

// Fragment-order copies (svla_flow_pack_weight) of the weights the persistent flow kernel reads: the expert
// layers' W8A16 linears as int8, the action / time projections as bf16.  Left empty (the flow loop then runs as
// per-layer launches) when the kernel cannot take the configuration or the engine was created with NO_FLOW.
int32_t pack_flow_weights(svla_engine* e, cudaStream_t stream) {
  const Cfg& c = e->cfg;
  if ((e->flags & SVLA_ENGINE_NO_FLOW) || c.chunk > SVLA_FLOW_MAX_ROWS || c.expert_layers > SVLA_FLOW_MAX_LAYERS ||
      c.expert_hidden % 16 || c.expert_hidden > 1024 || c.max_action_dim % 16 || c.expert_mlp % 16)
    return SVLA_OK;
  struct Job {
    std::string name;
    const void* w;
    int eb, n, k;
    int64_t ld;
  };
  std::vector<Job> jobs;
  const std::string ep = std::string(kExpert) + ".";
  for (const auto& kv : e->lin) {
    if (kv.first.compare(0, ep.size(), ep) != 0) continue;
    if (kv.second.kind != "w8a16") return SVLA_OK;  // the kernel reads int8 expert weights only
    jobs.push_back({kv.first, kv.second.weight, 1, kv.second.n, kv.second.k, kv.second.k});
  }
  const int E = c.expert_hidden;
  for (const char* n : {"model.action_in_proj", "model.action_time_mlp_out", "model.action_out_proj"}) {
    const Lin& l = e->lin.at(n);
    if (l.kind != "bf16") return SVLA_OK;
    jobs.push_back({n, l.weight, 2, l.n, l.k, l.k});
  }
  const Lin& ti = e->lin.at("model.action_time_mlp_in");  // its first E columns (the rest is a per-step constant)
  if (ti.kind != "bf16") return SVLA_OK;
  jobs.push_back({"model.action_time_mlp_in", ti.weight, 2, ti.n, E, ti.k});
  size_t total = 0;
  std::vector<size_t> off;
  for (const Job& j : jobs) {
    const size_t nb = svla_flow_packed_bytes(j.n, j.k, j.eb);
    if (nb == 0) return SVLA_OK;
    off.push_back(total);
    total += (nb + kAlign - 1) / kAlign * kAlign;
  }
  cudaError_t err = cudaMalloc(&e->flow_frag, total);
  if (err != cudaSuccess) {
    e->flow_frag = nullptr;
    return cuda_fail(err, "cudaMalloc(flow weights)");
  }
  for (size_t i = 0; i < jobs.size(); ++i) {
    const Job& j = jobs[i];
    const int32_t rc = svla_flow_pack_weight(j.w, j.eb, j.ld, j.n, j.k, e->flow_frag + off[i],
                                             reinterpret_cast<svla_stream_t>(stream));
    if (rc != SVLA_OK) return rc;
    e->frag[j.name] = e->flow_frag + off[i];
  }
  err = cudaStreamSynchronize(stream);
  return err == cudaSuccess ? SVLA_OK : cuda_fail(err, "packing the flow weights");
}

void release(svla_engine* e) {
  if (!e) return;
  cudaDeviceSynchronize();
  for (auto& kv : e->per_batch)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  if (e->capture_stream) cudaStreamDestroy(e->capture_stream);
  if (e->arena) cudaFree(e->arena);
  if (e->flow_frag) cudaFree(e->flow_frag);
  if (e->weights) cudaFree(e->weights);
  delete e;
}

PerBatch* launches_for(svla_engine* e, int B) {
  PerBatch& pb = e->per_batch[B];
  if (pb.launches.empty()) Builder(*e, B, &pb.launches).build();
  return &pb;
}

// copies rows of `cols` elements (elem bytes each) from src [rows, src_cols] into dst [rows, dst_cols]
cudaError_t copy_rows(void* dst, int dst_cols, const void* src, int src_cols, int cols, int rows, size_t elem,
                      cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  return cudaMemcpy2DAsync(dst, dst_cols * elem, src, src_cols * elem, cols * elem, rows, cudaMemcpyDefault, s);
}

}  // namespace engine_impl
}  // namespace svla

extern "C" {

int32_t svla_engine_inspect(const char* packed_path, svla_engine_info* info) {
  if (!info) return set_error(SVLA_ERR_ARG, "svla_engine_inspect: null info");
  PackedFile pf;
  std::string err;
  int32_t rc = read_header(packed_path, &pf, &err);
  if (rc == SVLA_OK) rc = check_tensors(pf, &err);
  if (rc != SVLA_OK) return set_error(rc, "svla_engine_inspect: " + err);
  fill_info(pf, info);
  return SVLA_OK;
}

int32_t svla_engine_create(const char* packed_path, int32_t max_batch, int32_t flags, svla_stream_t stream,
                           svla_engine** out) {
  if (!out) return set_error(SVLA_ERR_ARG, "svla_engine_create: null out");
  *out = nullptr;
  if (max_batch < 1 || max_batch > 4096) return set_error(SVLA_ERR_ARG, "svla_engine_create: max_batch must be 1..4096");
  if (flags & ~(SVLA_ENGINE_NO_GRAPH | SVLA_ENGINE_NO_SPLIT_K | SVLA_ENGINE_NO_FLOW))
    return set_error(SVLA_ERR_ARG, fmt("svla_engine_create: unknown flags 0x%x", flags));
  std::unique_ptr<svla_engine, void (*)(svla_engine*)> e(new svla_engine(), release);
  std::string err;
  int32_t rc = read_header(packed_path, &e->file, &err);
  if (rc == SVLA_OK) rc = check_tensors(e->file, &err);
  if (rc != SVLA_OK) return set_error(rc, "svla_engine_create: " + err);
  e->cfg = e->file.cfg;
  e->max_batch = max_batch;
  e->flags = flags;
  cudaError_t ce = cudaGetDevice(&e->device);
  if (ce != cudaSuccess) return cuda_fail(ce, "svla_engine_create: cudaGetDevice");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  rc = load_weights(e.get(), packed_path, s);
  if (rc != SVLA_OK) return rc;
  e->arena_bytes = layout_buffers(e->cfg, max_batch, nullptr, &e->buf);
  ce = cudaMalloc(&e->arena, e->arena_bytes);
  if (ce != cudaSuccess) {
    e->arena = nullptr;
    return cuda_fail(ce, "svla_engine_create: cudaMalloc(buffers)");
  }
  layout_buffers(e->cfg, max_batch, e->arena, &e->buf);
  // zeroed buffers: mask padding bytes read as 0 and the split-K tile counters start at zero
  ce = cudaMemsetAsync(e->arena, 0, e->arena_bytes, s);
  if (ce != cudaSuccess) return cuda_fail(ce, "svla_engine_create: clearing the buffers");
  rc = compute_constants(e.get(), s);
  if (rc != SVLA_OK) return rc;
  rc = pack_flow_weights(e.get(), s);
  if (rc != SVLA_OK) return rc;
  ce = cudaStreamCreateWithFlags(&e->capture_stream, cudaStreamNonBlocking);
  if (ce != cudaSuccess) return cuda_fail(ce, "svla_engine_create: cudaStreamCreate");
  e->launches_per_call = static_cast<int>(launches_for(e.get(), max_batch)->launches.size());
  *out = e.release();
  return SVLA_OK;
}

int32_t svla_engine_get_info(const svla_engine* engine, svla_engine_info* info) {
  if (!engine || !info) return set_error(SVLA_ERR_ARG, "svla_engine_get_info: null argument");
  fill_info(engine->file, info);
  info->max_batch = engine->max_batch;
  info->launches_per_call = engine->launches_per_call;
  info->buffer_bytes = static_cast<int64_t>(engine->arena_bytes);
  return SVLA_OK;
}

int32_t svla_engine_sample_actions(svla_engine* e, const float* const* images, const uint8_t* const* img_masks,
                                   const int64_t* lang_tokens, const uint8_t* lang_masks, int32_t lang_len,
                                   const float* state, int32_t state_dim, const float* noise, int32_t batch,
                                   float* actions, svla_stream_t stream) {
  if (!e) return set_error(SVLA_ERR_ARG, "svla_engine_sample_actions: null engine");
  const Cfg& c = e->cfg;
  if (batch < 1 || batch > e->max_batch)
    return set_error(SVLA_ERR_ARG, fmt("svla_engine_sample_actions: batch %d outside 1..%d", batch, e->max_batch));
  if (!images || !img_masks || !lang_tokens || !lang_masks || !state || !noise || !actions)
    return set_error(SVLA_ERR_ARG, "svla_engine_sample_actions: null input or output");
  for (int cam = 0; cam < c.n_cams; ++cam)
    if (!images[cam] || !img_masks[cam]) return set_error(SVLA_ERR_ARG, "svla_engine_sample_actions: null camera");
  if (lang_len < 0 || state_dim < 0 || state_dim > c.max_state_dim)
    return set_error(SVLA_ERR_ARG, fmt("svla_engine_sample_actions: lang_len %d / state_dim %d (max %d)", lang_len,
                                       state_dim, c.max_state_dim));
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev != e->device)
    return set_error(SVLA_ERR_ARG, fmt("svla_engine_sample_actions: engine lives on device %d, current is %d",
                                       e->device, dev));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const Buffers& b = e->buf;
  const int B = batch, S = c.chunk, A = c.max_action_dim;
  const size_t img = static_cast<size_t>(c.channels) * c.image_size * c.image_size;
  cudaError_t ce = cudaSuccess;
  // inputs -> the static buffers (images interleaved by camera: [B, n_cams, C, S, S])
  for (int cam = 0; cam < c.n_cams && ce == cudaSuccess; ++cam) {
    ce = cudaMemcpy2DAsync(b.in_img + cam * img, c.n_cams * img * 4, images[cam], img * 4, img * 4, B,
                           cudaMemcpyDefault, s);
    if (ce == cudaSuccess) ce = cudaMemcpyAsync(b.in_img_mask + static_cast<size_t>(cam) * B, img_masks[cam], B,
                                                cudaMemcpyDefault, s);
  }
  const int nl = lang_len < c.n_lang ? lang_len : c.n_lang;
  if (ce == cudaSuccess && nl < c.n_lang) {
    ce = cudaMemsetAsync(b.in_tokens, 0, static_cast<size_t>(B) * c.n_lang * 8, s);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(b.in_lang_mask, 0, static_cast<size_t>(B) * c.n_lang, s);
  }
  if (ce == cudaSuccess) ce = copy_rows(b.in_tokens, c.n_lang, lang_tokens, lang_len, nl, B, 8, s);
  if (ce == cudaSuccess) ce = copy_rows(b.in_lang_mask, c.n_lang, lang_masks, lang_len, nl, B, 1, s);
  if (ce == cudaSuccess && state_dim < c.max_state_dim)
    ce = cudaMemsetAsync(b.in_state, 0, static_cast<size_t>(B) * c.max_state_dim * 4, s);
  if (ce == cudaSuccess) ce = copy_rows(b.in_state, c.max_state_dim, state, state_dim, state_dim, B, 4, s);
  if (ce == cudaSuccess)
    ce = cudaMemcpyAsync(b.in_noise, noise, static_cast<size_t>(B) * S * A * 4, cudaMemcpyDefault, s);
  if (ce != cudaSuccess) return cuda_fail(ce, "svla_engine_sample_actions: input copy");
  PerBatch* pb = launches_for(e, B);
  if (pb->exec) {
    ce = cudaGraphLaunch(pb->exec, s);
    if (ce != cudaSuccess) return cuda_fail(ce, "svla_engine_sample_actions: cudaGraphLaunch");
  } else {
    const int32_t rc = run_list(pb->launches, s);
    if (rc != SVLA_OK) return rc;
    ++pb->runs;
    if (!(e->flags & SVLA_ENGINE_NO_GRAPH)) {
      // record the list after its first (eager) run, which did the kernels' one-time host set-up
      cudaGraph_t g = nullptr;
      ce = cudaStreamBeginCapture(e->capture_stream, cudaStreamCaptureModeThreadLocal);
      if (ce != cudaSuccess) return cuda_fail(ce, "svla_engine_sample_actions: cudaStreamBeginCapture");
      const int32_t crc = run_list(pb->launches, e->capture_stream);
      ce = cudaStreamEndCapture(e->capture_stream, &g);
      if (crc != SVLA_OK) {
        if (g) cudaGraphDestroy(g);
        return crc;
      }
      if (ce != cudaSuccess) return cuda_fail(ce, "svla_engine_sample_actions: cudaStreamEndCapture");
      ce = cudaGraphInstantiate(&pb->exec, g, 0);
      cudaGraphDestroy(g);
      if (ce != cudaSuccess) {
        pb->exec = nullptr;
        return cuda_fail(ce, "svla_engine_sample_actions: cudaGraphInstantiate");
      }
    }
  }
  ce = cudaMemcpyAsync(actions, b.xt, static_cast<size_t>(B) * S * A * 4, cudaMemcpyDefault, s);
  if (ce != cudaSuccess) return cuda_fail(ce, "svla_engine_sample_actions: output copy");
  return SVLA_OK;
}

int32_t svla_engine_destroy(svla_engine* engine) {
  release(engine);
  return SVLA_OK;
}

}  // extern "C"
