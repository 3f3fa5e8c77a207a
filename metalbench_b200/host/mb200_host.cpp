// mb200_host — drop-in for the reference's build/metalbench_host.
//
//   mb200_host --manifest m.json
//
// Reads the manifest the reference harness writes (mlx/scripts/mlx_helpers.py
// build_manifest, lines 290-335: function, metallib, buffers[{binding, role:
// input|output|scalar, path, size, dtype, value}], grid, threadgroup, warmup,
// iters, profile, capture_path), runs the kernel through libmb200's mb_run and
// prints ONE JSON line with the keys of metal/scripts/main.mm:184-195 (chip,
// metal_device, tg_static_mem_bytes, pso_max_threads_per_tg, min_ms,
// median_ms, mean_ms, iters, available_counter_sets, profiling). Outputs are
// written to their `path`. Banners go to stderr; any error prints a message
// and exits 1, like main.mm's die().
//
// Extensions: buffer "dtype" ("f32" default, "bf16", "i32", "u32") for inputs
// and outputs, a top-level "kernel" (libmb200 name; otherwise "function" is
// mapped from the reference's Metal function name) and "config" (object
// passed to mb_run as its config JSON). grid/threadgroup are accepted and
// ignored: every CUDA kernel chooses its own launch shape.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "mb200.h"

namespace {

// ---- minimal JSON value + parser ------------------------------------------
struct J {
  enum T { NUL, BOOL, NUM, STR, ARR, OBJ } t = NUL;
  bool b = false;
  double n = 0;
  std::string s;
  std::vector<J> a;
  std::vector<std::pair<std::string, J>> o;
  const J* get(const char* k) const {
    for (auto& kv : o)
      if (kv.first == k) return &kv.second;
    return nullptr;
  }
};

struct Parser {
  const char* p;
  const char* end;
  std::string err;
  void ws() {
    while (p < end && (*p == ' ' || *p == '\n' || *p == '\t' || *p == '\r')) ++p;
  }
  bool lit(const char* w) {
    size_t n = strlen(w);
    if ((size_t)(end - p) >= n && !strncmp(p, w, n)) {
      p += n;
      return true;
    }
    return false;
  }
  bool str(std::string& out) {
    if (p >= end || *p != '"') return false;
    ++p;
    while (p < end && *p != '"') {
      if (*p == '\\' && p + 1 < end) {
        ++p;
        switch (*p) {
          case 'n': out += '\n'; break;
          case 't': out += '\t'; break;
          case 'r': out += '\r'; break;
          case 'b': out += '\b'; break;
          case 'f': out += '\f'; break;
          case 'u': {  // keep BMP code points < 0x80, replace the rest
            if (end - p < 5) return false;
            unsigned v = (unsigned)strtoul(std::string(p + 1, p + 5).c_str(), nullptr, 16);
            out += v < 0x80 ? (char)v : '?';
            p += 4;
            break;
          }
          default: out += *p;
        }
        ++p;
      } else {
        out += *p++;
      }
    }
    if (p >= end) return false;
    ++p;
    return true;
  }
  bool val(J& v) {
    ws();
    if (p >= end) return false;
    if (*p == '{') {
      v.t = J::OBJ;
      ++p;
      ws();
      if (p < end && *p == '}') { ++p; return true; }
      while (true) {
        ws();
        std::string k;
        if (!str(k)) return false;
        ws();
        if (p >= end || *p != ':') return false;
        ++p;
        J c;
        if (!val(c)) return false;
        v.o.emplace_back(k, c);
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == '}') { ++p; return true; }
        return false;
      }
    }
    if (*p == '[') {
      v.t = J::ARR;
      ++p;
      ws();
      if (p < end && *p == ']') { ++p; return true; }
      while (true) {
        J c;
        if (!val(c)) return false;
        v.a.push_back(c);
        ws();
        if (p < end && *p == ',') { ++p; continue; }
        if (p < end && *p == ']') { ++p; return true; }
        return false;
      }
    }
    if (*p == '"') { v.t = J::STR; return str(v.s); }
    if (lit("true")) { v.t = J::BOOL; v.b = true; return true; }
    if (lit("false")) { v.t = J::BOOL; v.b = false; return true; }
    if (lit("null")) { v.t = J::NUL; return true; }
    char* e = nullptr;
    v.n = strtod(p, &e);
    if (e == p) return false;
    v.t = J::NUM;
    p = e;
    return true;
  }
};

std::string dump(const J& v) {  // flat re-serialisation for the mb_run config
  char buf[64];
  switch (v.t) {
    case J::NUL: return "null";
    case J::BOOL: return v.b ? "true" : "false";
    case J::NUM: snprintf(buf, sizeof buf, "%.17g", v.n); return buf;
    case J::STR: return "\"" + v.s + "\"";
    case J::ARR: {
      std::string s = "[";
      for (size_t i = 0; i < v.a.size(); ++i) s += (i ? "," : "") + dump(v.a[i]);
      return s + "]";
    }
    case J::OBJ: {
      std::string s = "{";
      for (size_t i = 0; i < v.o.size(); ++i)
        s += (i ? ",\"" : "\"") + v.o[i].first + "\":" + dump(v.o[i].second);
      return s + "}";
    }
  }
  return "null";
}

int die(const std::string& msg) {
  fprintf(stderr, "[host] error: %s\n", msg.c_str());
  return 1;
}

bool read_file(const std::string& path, std::vector<char>& out) {
  FILE* f = fopen(path.c_str(), "rb");
  if (!f) return false;
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  out.resize(n > 0 ? (size_t)n : 0);
  bool ok = n <= 0 || fread(out.data(), 1, (size_t)n, f) == (size_t)n;
  fclose(f);
  return ok;
}

int dtype_tag(const std::string& d) {
  if (d == "f32") return MB_F32;
  if (d == "bf16") return MB_BF16;
  if (d == "f16") return MB_F16;
  if (d == "i32") return MB_I32;
  if (d == "u32") return MB_U32;
  return -1;
}

// The reference's Metal function names of the hot-path kernels -> libmb200.
// (The standard- and full-set kernels take bf16 buffers: manifests for them
// set "dtype": "bf16", an extension of the reference's f32/f16/i32/u32.)
const std::map<std::string, std::string> kFunctionToKernel = {
    {"sqr_matmul_f32", "sqr_mm"},
    {"rect_matmul_f32", "sqr_mm"},
    {"batch_matmul_f32", "batch_mm"},
    {"transpose_2d_f32", "transpose_2d"},
    {"conv2d_f32", "conv2d"},
    {"llama_decoder_layer_f32", "llama_decoder_layer"},
    {"rms_norm_linear_f32", "rms_norm_linear"},
    {"fused_add_rms_norm_f32", "fused_add_rms_norm"},
    {"rope_embedding_f32", "rope_embedding"},
    {"swiglu_f32", "swiglu"},
    {"fused_qkv_projection_f32", "gemm_bf16"},
    {"scaled_dot_product_f32", "scaled_dot_product"},
    {"llama_attention_f32", "llama_attention"},
    {"mha_attention_f32", "mha_attention"},
    {"transformer_block_f32", "transformer_block"},
};

std::string json_escape(const char* s) {
  std::string o;
  for (; *s; ++s) {
    if (*s == '"' || *s == '\\') o += '\\';
    o += *s;
  }
  return o;
}

}  // namespace

int main(int argc, char** argv) {
  const char* mpath = nullptr;
  for (int i = 1; i + 1 < argc; ++i)
    if (!strcmp(argv[i], "--manifest")) mpath = argv[i + 1];
  if (!mpath) return die("missing --manifest <path>");
  std::vector<char> text;
  if (!read_file(mpath, text)) return die("cannot read manifest");
  Parser ps{text.data(), text.data() + text.size(), {}};
  J m;
  if (!ps.val(m) || m.t != J::OBJ) return die("manifest json parse");

  int dev = 0;
  if (const char* e = getenv("LOCAL_RANK")) dev = atoi(e);
  if (mb_init(dev, 0, 1, nullptr, 0) != MB_OK) return die(mb_last_error());
  mb_device d;
  if (mb_device_info(&d) != MB_OK) return die(mb_last_error());
  fprintf(stderr, "[host] %s (%s) | %d CPU | %d SM | %.0f GB HBM\n", d.name, d.type, d.cpu_cores,
          d.sm_count, d.hbm_bytes / 1e9);

  std::string kernel;
  if (const J* k = m.get("kernel")) kernel = k->s;
  if (kernel.empty()) {
    const J* f = m.get("function");
    if (!f) return die("manifest has neither kernel nor function");
    auto it = kFunctionToKernel.find(f->s);
    kernel = it == kFunctionToKernel.end() ? f->s : it->second;
  }
  const J* bl = m.get("buffers");
  if (!bl || bl->t != J::ARR) return die("manifest buffers missing");

  std::vector<mb_buf> bufs;
  std::vector<mb_scalar> scalars;
  std::vector<std::unique_ptr<std::vector<char>>> store;
  std::vector<std::pair<std::string, size_t>> outs;  // path, index into store
  for (const J& b : bl->a) {
    const J* role = b.get("role");
    const J* bind = b.get("binding");
    if (!role || !bind) return die("buffer without role/binding");
    const J* dt = b.get("dtype");
    const std::string dts = dt ? dt->s : "f32";
    if (role->s == "input" || role->s == "output") {
      const int tag = dtype_tag(dts);
      if (tag < 0) return die("unknown buffer dtype " + dts);
      const J* path = b.get("path");
      if (!path) return die("buffer without path");
      store.emplace_back(new std::vector<char>());
      std::vector<char>& data = *store.back();
      if (role->s == "input") {
        if (!read_file(path->s, data)) return die("cannot read input " + path->s);
      } else {
        const J* sz = b.get("size");
        if (!sz) return die("output without size");
        data.resize((size_t)sz->n);
        outs.emplace_back(path->s, store.size() - 1);
      }
      mb_buf mbb{(int)bind->n, role->s == "input" ? MB_ROLE_INPUT : MB_ROLE_OUTPUT, tag, 0,
                 data.data(), data.size()};
      bufs.push_back(mbb);
    } else if (role->s == "scalar") {
      mb_scalar s;
      s.binding = (int)bind->n;
      const J* v = b.get("value");
      const double x = v ? v->n : 0;
      if (dts == "f32") { s.dtype = MB_F32; s.v.f = (float)x; }
      else if (dts == "i32") { s.dtype = MB_I32; s.v.i = (int32_t)x; }
      else if (dts == "u32") { s.dtype = MB_U32; s.v.u = (uint32_t)x; }
      else return die("unknown scalar dtype " + dts);
      scalars.push_back(s);
    } else {
      return die("unknown buffer role " + role->s);
    }
  }
  const J* w = m.get("warmup");
  const J* it = m.get("iters");
  const int warmup = w ? (int)w->n : 10, iters = it ? (int)it->n : 100;
  std::string cfg = "{}";
  if (const J* c = m.get("config")) cfg = dump(*c);
  const J* prof = m.get("profile");
  const bool profile = prof && (prof->t == J::BOOL ? prof->b : prof->n != 0);
  if (profile) {  // the manifest's profile flag rides in the config object
    if (cfg.size() > 2)
      cfg = cfg.substr(0, cfg.size() - 1) + ",\"profile\":true}";
    else
      cfg = "{\"profile\":true}";
  }
  fprintf(stderr, "[host] kernel `%s` | setup complete\n", kernel.c_str());

  mb_timing t;
  memset(&t, 0, sizeof t);
  if (mb_run(kernel.c_str(), bufs.data(), (int)bufs.size(), scalars.data(), (int)scalars.size(),
             cfg.c_str(), warmup, iters, &t) != MB_OK)
    return die(mb_last_error());
  for (auto& o : outs) {
    FILE* f = fopen(o.first.c_str(), "wb");
    const std::vector<char>& data = *store[o.second];
    if (!f || fwrite(data.data(), 1, data.size(), f) != data.size()) {
      if (f) fclose(f);
      return die("cannot write output " + o.first);
    }
    fclose(f);
  }
  printf(
      "{\"chip\":{\"type\":\"%s\",\"name\":\"%s\",\"bucket\":\"%s\",\"cpu_cores\":%d,"
      "\"gpu_cores\":%d,\"ram_bytes\":%llu},\"metal_device\":\"%s\",\"device\":\"%s\","
      "\"tg_static_mem_bytes\":%d,\"pso_max_threads_per_tg\":%d,"
      "\"min_ms\":%.6f,\"median_ms\":%.6f,\"mean_ms\":%.6f,\"iters\":%d,"
      "\"available_counter_sets\":[],\"profiling\":{\"counters_available\":false,"
      "\"enabled\":%s,\"profile_ms\":%.6f,\"nvtx_range\":\"mb_profile:%s\"}}\n",
      d.type, json_escape(d.name).c_str(), d.bucket, d.cpu_cores, d.sm_count,
      (unsigned long long)d.ram_bytes, json_escape(d.name).c_str(), json_escape(d.name).c_str(),
      t.smem_bytes, t.threads_per_cta, t.min_ms, t.median_ms, t.mean_ms, t.iters,
      profile ? "true" : "false", t.profile_ms, json_escape(kernel.c_str()).c_str());
  mb_shutdown();
  return 0;
}
