// Node-API addon over include/gsampler.h: the reference engine's sampleToken
// (src/runtime/sampling.ts:18-65), called at src/runtime/gemma-session.ts:686, 705 and 1328,
// runs on the B200 through gs_sample_host.  Built with node-gyp (binding.gyp beside this
// file) against libgsampler.so; sampling-gpu.ts is the TypeScript side.
//
//   sampleHost(logits: Float32Array, historyIds: Int32Array, historyCounts: Int32Array,
//              config: DecodingConfig, uniform: number, softcap?: number): number
//
// `historyIds` / `historyCounts`: the repetition window as its distinct ids in order of
// first occurrence and the occurrences of each (gs_batch.history_count), so a window of
// any length fits.  `uniform`: the value of the caller's random() (drawn by the shim only
// when temperature != 0, as the reference draws it).  Errors are thrown with the
// reference's messages.
#include <node_api.h>

#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <string>

#include "gsampler.h"

namespace {

// One gs_ctx per Node environment (the main thread and each worker thread), kept as the
// environment's instance data and destroyed with it.
void destroy_ctx(napi_env, void* data, void*) {
  if (data) gs_destroy(static_cast<gs_ctx*>(data));
}

gs_ctx* env_ctx(napi_env env, gs_status* st) {
  void* data = nullptr;
  *st = GS_OK;
  if (napi_get_instance_data(env, &data) == napi_ok && data) return static_cast<gs_ctx*>(data);
  const char* dev = std::getenv("GS_DEVICE");
  gs_ctx* c = nullptr;
  *st = gs_create(dev ? std::atoi(dev) : 0, &c);
  if (*st != GS_OK) return nullptr;
  napi_set_instance_data(env, c, destroy_ctx, nullptr);
  return c;
}

napi_value throw_error(napi_env env, const std::string& msg) {
  napi_throw_error(env, nullptr, msg.c_str());
  return nullptr;
}

bool typed(napi_env env, napi_value v, napi_typedarray_type want, void** data, size_t* len) {
  bool is = false;
  if (napi_is_typedarray(env, v, &is) != napi_ok || !is) return false;
  napi_typedarray_type t;
  napi_value ab;
  size_t off = 0;
  if (napi_get_typedarray_info(env, v, &t, len, data, &ab, &off) != napi_ok) return false;
  return t == want;
}

double number_prop(napi_env env, napi_value obj, const char* key, bool* ok) {
  napi_value v;
  double d = 0.0;
  if (napi_get_named_property(env, obj, key, &v) != napi_ok || napi_get_value_double(env, v, &d) != napi_ok) *ok = false;
  return d;
}

// (the row flags of a sampled row, as the reference's errors)
const char* flag_error(uint32_t fl) {
  if (fl & GS_FLAG_ERR_DEADEND) return "Generation constraint reached a tokenization dead end";
  if (fl & GS_FLAG_ERR_NONFINITE) return "logits contain NaN or +Infinity";
  if (fl & GS_FLAG_ERR_INVALID) return "mask state out of range";
  if (fl & GS_FLAG_ERR_UNSUPPORTED) return "request outside the implemented envelope";
  if (fl & GS_FLAG_ERR_TIMEOUT) return "device wait timed out";
  return nullptr;
}

napi_value SampleHost(napi_env env, napi_callback_info info) {
  size_t argc = 6;
  napi_value argv[6];
  if (napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr) != napi_ok || argc < 5)
    return throw_error(env, "sampleHost(logits, historyIds, historyCounts, config, uniform[, softcap])");
  void* logits = nullptr;
  size_t vocab = 0;
  if (!typed(env, argv[0], napi_float32_array, &logits, &vocab)) return throw_error(env, "logits must be a Float32Array");
  if (vocab == 0) return throw_error(env, "Cannot sample empty logits");
  void* ids = nullptr;
  void* counts = nullptr;
  size_t n_ids = 0, n_counts = 0;
  if (!typed(env, argv[1], napi_int32_array, &ids, &n_ids) || !typed(env, argv[2], napi_int32_array, &counts, &n_counts) ||
      n_ids != n_counts)
    return throw_error(env, "historyIds and historyCounts must be Int32Arrays of one length");
  if (n_ids > GS_MAX_HISTORY) return throw_error(env, "repetition window holds more than 4096 distinct ids");
  bool ok = true;
  gs_params p{};
  p.temperature = number_prop(env, argv[3], "temperature", &ok);
  p.top_p = number_prop(env, argv[3], "topP", &ok);
  p.min_p = number_prop(env, argv[3], "minP", &ok);
  p.typical_p = number_prop(env, argv[3], "typicalP", &ok);
  p.repetition_penalty = number_prop(env, argv[3], "repetitionPenalty", &ok);
  p.presence_penalty = number_prop(env, argv[3], "presencePenalty", &ok);
  p.frequency_penalty = number_prop(env, argv[3], "frequencyPenalty", &ok);
  const double top_k = number_prop(env, argv[3], "topK", &ok);
  if (!ok) return throw_error(env, "config must hold the DecodingConfig numbers");
  // (gs_params.top_k is an int32: a topK that is not a non-negative integer is refused
  // here with validateDecodingConfig's message, src/runtime/decoding.ts:35; the other
  // fields are checked by the library)
  if (!(top_k >= 0.0 && std::isfinite(top_k) && std::floor(top_k) == top_k))
    return throw_error(env, "topK must be a non-negative integer");
  // topK beyond int32 keeps the whole vocabulary, as topK >= vocab does in the reference
  p.top_k = top_k > 2147483647.0 ? 2147483647 : static_cast<int32_t>(top_k);
  double uniform = 0.0;
  if (napi_get_value_double(env, argv[4], &uniform) != napi_ok) return throw_error(env, "uniform must be a number");
  double softcap = 0.0;
  if (argc > 5) napi_get_value_double(env, argv[5], &softcap);

  gs_status cs = GS_OK;
  gs_ctx* ctx = env_ctx(env, &cs);
  if (!ctx) return throw_error(env, "gs_create failed (status " + std::to_string(cs) + ")");
  int32_t hlen = static_cast<int32_t>(n_ids);
  gs_batch b{};
  b.logits = logits;
  b.dtype = GS_DTYPE_F32;
  b.rows = 1;
  b.vocab = static_cast<int64_t>(vocab);
  b.row_stride = static_cast<int64_t>(vocab);
  b.softcap = static_cast<float>(softcap);
  b.params_count = 1;
  b.params = &p;
  if (n_ids > 0) {
    b.history = static_cast<const int32_t*>(ids);
    b.history_len = &hlen;
    b.history_stride = static_cast<int64_t>(n_ids);
    b.history_count = static_cast<const int32_t*>(counts);
  }
  b.uniforms = &uniform;  // (not read for temperature 0: no draw)
  int32_t id = -1;
  uint32_t flags = 0;
  gs_outputs o{};
  o.ids = &id;
  o.flags = &flags;
  const gs_status s = gs_sample_host(ctx, &b, &o, nullptr);
  if (s == GS_EEMPTY) return throw_error(env, "Cannot sample empty logits");
  if (s != GS_OK) {
    const char* m = gs_last_error(ctx);
    return throw_error(env, m && *m ? m : "gs_sample_host failed (status " + std::to_string(s) + ")");
  }
  if (const char* m = flag_error(flags)) return throw_error(env, m);
  napi_value out;
  napi_create_int32(env, id, &out);
  return out;
}

napi_value Init(napi_env env, napi_value exports) {
  napi_value fn;
  napi_create_function(env, "sampleHost", NAPI_AUTO_LENGTH, SampleHost, nullptr, &fn);
  napi_set_named_property(env, exports, "sampleHost", fn);
  return exports;
}

}  // namespace

NAPI_MODULE(NODE_GYP_MODULE_NAME, Init)
