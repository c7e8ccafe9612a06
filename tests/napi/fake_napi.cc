// Test harness for the Node-API addon (gemma-webgpu-engine_b200/node/gsampler_napi.cc):
// a minimal Node-API runtime (numbers, objects with named properties, Float32Array /
// Int32Array, functions, thrown errors) and a driver that loads the addon's exports and
// calls sampleHost once with inputs read from a binary file:
//   int64 vocab, float32[vocab] logits, int64 n, int32[n] ids, int32[n] counts,
//   float64[8] temperature topP minP typicalP repetitionPenalty presencePenalty
//   frequencyPenalty topK, float64 uniform, float64 softcap
// It prints "id <token>" or "error <message>".
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "node_api.h"

struct napi_value__ {
  int kind = 0;  // 0 number, 1 object, 2 typed array, 3 function
  double num = 0.0;
  std::map<std::string, napi_value> props;
  napi_typedarray_type ta = napi_float32_array;
  void* data = nullptr;
  size_t len = 0;
  napi_callback fn = nullptr;
};
struct napi_env__ {
  std::vector<std::unique_ptr<napi_value__>> values;
  std::string error;
  bool thrown = false;
  void* instance = nullptr;
  napi_finalize instance_fin = nullptr;
  napi_value make() {
    values.emplace_back(new napi_value__());
    return values.back().get();
  }
};
struct napi_callback_info__ {
  std::vector<napi_value> args;
};

extern "C" {
napi_status napi_get_cb_info(napi_env, napi_callback_info info, size_t* argc, napi_value* argv, napi_value*, void**) {
  const size_t n = *argc;
  for (size_t i = 0; i < n; ++i) argv[i] = i < info->args.size() ? info->args[i] : nullptr;
  *argc = info->args.size();
  return napi_ok;
}
napi_status napi_is_typedarray(napi_env, napi_value v, bool* r) {
  *r = v && v->kind == 2;
  return napi_ok;
}
napi_status napi_get_typedarray_info(napi_env, napi_value v, napi_typedarray_type* t, size_t* len, void** data,
                                     napi_value* ab, size_t* off) {
  *t = v->ta;
  *len = v->len;
  *data = v->data;
  *ab = nullptr;
  *off = 0;
  return napi_ok;
}
napi_status napi_get_named_property(napi_env, napi_value o, const char* k, napi_value* r) {
  auto it = o->props.find(k);
  if (it == o->props.end()) return static_cast<napi_status>(1);
  *r = it->second;
  return napi_ok;
}
napi_status napi_set_named_property(napi_env, napi_value o, const char* k, napi_value v) {
  o->props[k] = v;
  return napi_ok;
}
napi_status napi_get_value_double(napi_env, napi_value v, double* r) {
  if (!v || v->kind != 0) return static_cast<napi_status>(1);
  *r = v->num;
  return napi_ok;
}
napi_status napi_create_int32(napi_env env, int32_t x, napi_value* r) {
  *r = env->make();
  (*r)->num = x;
  return napi_ok;
}
napi_status napi_throw_error(napi_env env, const char*, const char* msg) {
  env->thrown = true;
  env->error = msg ? msg : "";
  return napi_ok;
}
napi_status napi_create_function(napi_env env, const char*, size_t, napi_callback cb, void*, napi_value* r) {
  *r = env->make();
  (*r)->kind = 3;
  (*r)->fn = cb;
  return napi_ok;
}
napi_status napi_set_instance_data(napi_env env, void* data, napi_finalize fin, void*) {
  env->instance = data;
  env->instance_fin = fin;
  return napi_ok;
}
napi_status napi_get_instance_data(napi_env env, void** data) {
  *data = env->instance;
  return napi_ok;
}
napi_value napi_register_module_v1(napi_env, napi_value);
}

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  FILE* f = std::fopen(argv[1], "rb");
  if (!f) return 2;
  auto rd = [&](void* p, size_t n) { return std::fread(p, 1, n, f) == n; };
  int64_t vocab = 0, n = 0;
  bool ok = rd(&vocab, 8);
  std::vector<float> logits(static_cast<size_t>(vocab));
  ok = ok && (vocab == 0 || rd(logits.data(), 4 * logits.size())) && rd(&n, 8);
  std::vector<int32_t> ids(static_cast<size_t>(n)), counts(static_cast<size_t>(n));
  double cfg[8], uniform = 0.0, softcap = 0.0;
  ok = ok && (n == 0 || (rd(ids.data(), 4 * ids.size()) && rd(counts.data(), 4 * counts.size()))) && rd(cfg, 64) &&
       rd(&uniform, 8) && rd(&softcap, 8);
  std::fclose(f);
  if (!ok) return 2;

  napi_env__ env;
  napi_value exports = env.make();
  exports->kind = 1;
  napi_register_module_v1(&env, exports);
  napi_value fn = exports->props.at("sampleHost");
  auto typed = [&](napi_typedarray_type t, void* data, size_t len) {
    napi_value v = env.make();
    v->kind = 2;
    v->ta = t;
    v->data = data;
    v->len = len;
    return v;
  };
  auto number = [&](double x) {
    napi_value v = env.make();
    v->num = x;
    return v;
  };
  napi_value config = env.make();
  config->kind = 1;
  const char* keys[8] = {"temperature", "topP", "minP", "typicalP", "repetitionPenalty", "presencePenalty",
                         "frequencyPenalty", "topK"};
  for (int i = 0; i < 8; ++i) config->props[keys[i]] = number(cfg[i]);
  napi_callback_info__ info;
  info.args = {typed(napi_float32_array, logits.data(), logits.size()), typed(napi_int32_array, ids.data(), ids.size()),
               typed(napi_int32_array, counts.data(), counts.size()), config, number(uniform), number(softcap)};
  napi_value r = fn->fn(&env, &info);
  if (env.thrown) {
    std::printf("error %s\n", env.error.c_str());
  } else {
    std::printf("id %d\n", static_cast<int>(r->num));
  }
  if (env.instance_fin) env.instance_fin(&env, env.instance, nullptr);  // (the environment's teardown)
  return 0;
}
