// Test stand-in for Node's node_api.h: the Node-API declarations the addon
// (gemma-webgpu-engine_b200/node/gsampler_napi.cc) uses, written from the public Node-API
// documentation, so that the addon builds here (no Node in this image) and runs against
// tests/napi/fake_napi.cc.  A real build uses Node's own header through node-gyp.
#pragma once
#include <cstddef>
#include <cstdint>
typedef struct napi_env__* napi_env;
typedef struct napi_value__* napi_value;
typedef struct napi_callback_info__* napi_callback_info;
typedef enum { napi_ok } napi_status;
typedef enum { napi_int8_array, napi_uint8_array, napi_uint8_clamped_array, napi_int16_array, napi_uint16_array,
               napi_int32_array, napi_uint32_array, napi_float32_array, napi_float64_array } napi_typedarray_type;
typedef napi_value (*napi_callback)(napi_env, napi_callback_info);
typedef void (*napi_finalize)(napi_env, void*, void*);
#define NAPI_AUTO_LENGTH SIZE_MAX
extern "C" {
napi_status napi_get_cb_info(napi_env, napi_callback_info, size_t*, napi_value*, napi_value*, void**);
napi_status napi_is_typedarray(napi_env, napi_value, bool*);
napi_status napi_get_typedarray_info(napi_env, napi_value, napi_typedarray_type*, size_t*, void**, napi_value*, size_t*);
napi_status napi_get_named_property(napi_env, napi_value, const char*, napi_value*);
napi_status napi_set_named_property(napi_env, napi_value, const char*, napi_value);
napi_status napi_get_value_double(napi_env, napi_value, double*);
napi_status napi_create_int32(napi_env, int32_t, napi_value*);
napi_status napi_throw_error(napi_env, const char*, const char*);
napi_status napi_create_function(napi_env, const char*, size_t, napi_callback, void*, napi_value*);
napi_status napi_set_instance_data(napi_env, void*, napi_finalize, void*);
napi_status napi_get_instance_data(napi_env, void**);
}
#define NAPI_MODULE(name, init) extern "C" napi_value napi_register_module_v1(napi_env e, napi_value x) { return init(e, x); }
#define NODE_GYP_MODULE_NAME gsampler
