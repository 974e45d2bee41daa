"""CPU checks of the Node integration sources (textsift_b200/node/): node is
not installed here, so the addon cannot be built or loaded; instead

  * the N-API C glue type-checks against include/textsift_cuda.h (gcc
    -fsyntax-only with a minimal stand-in for node_api.h that declares the
    N-API calls it makes, with their documented signatures);
  * every library function it calls is declared in the header;
  * the TypeScript CudaBackend's CudaApi interface names exactly the functions
    the addon registers, and the class calls nothing else.
"""
import os
import re
import subprocess

from conftest import ROOT

NODE = os.path.join(ROOT, "textsift_b200", "node")
C_SRC = os.path.join(NODE, "textsift_cuda_napi.c")
TS_SRC = os.path.join(NODE, "cuda-backend.ts")
HEADER = os.path.join(ROOT, "include", "textsift_cuda.h")

# A stand-in for node_api.h with the declarations the glue uses (N-API's
# documented C signatures); enough for a syntax and type check.
NODE_API_STUB = r"""
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>
typedef struct napi_env__* napi_env;
typedef struct napi_value__* napi_value;
typedef struct napi_callback_info__* napi_callback_info;
typedef enum { napi_ok, napi_invalid_arg, napi_generic_failure } napi_status;
typedef enum { napi_undefined, napi_null, napi_boolean, napi_number, napi_string, napi_symbol, napi_object,
               napi_function, napi_external, napi_bigint } napi_valuetype;
typedef enum { napi_int8_array, napi_uint8_array, napi_uint8_clamped_array, napi_int16_array, napi_uint16_array,
               napi_int32_array, napi_uint32_array, napi_float32_array, napi_float64_array, napi_bigint64_array,
               napi_biguint64_array } napi_typedarray_type;
typedef enum { napi_default = 0 } napi_property_attributes;
typedef napi_value (*napi_callback)(napi_env env, napi_callback_info info);
typedef struct { const char* utf8name; napi_value name; napi_callback method; napi_callback getter;
                 napi_callback setter; napi_value value; napi_property_attributes attributes; void* data;
               } napi_property_descriptor;
#define NAPI_AUTO_LENGTH SIZE_MAX
napi_status napi_throw_error(napi_env env, const char* code, const char* msg);
napi_status napi_get_undefined(napi_env env, napi_value* result);
napi_status napi_get_cb_info(napi_env env, napi_callback_info cbinfo, size_t* argc, napi_value* argv,
                             napi_value* this_arg, void** data);
napi_status napi_typeof(napi_env env, napi_value value, napi_valuetype* result);
napi_status napi_get_value_bigint_uint64(napi_env env, napi_value value, uint64_t* result, bool* lossless);
napi_status napi_create_bigint_uint64(napi_env env, uint64_t value, napi_value* result);
napi_status napi_is_typedarray(napi_env env, napi_value value, bool* result);
napi_status napi_get_typedarray_info(napi_env env, napi_value typedarray, napi_typedarray_type* type,
                                     size_t* length, void** data, napi_value* arraybuffer, size_t* byte_offset);
napi_status napi_get_value_uint32(napi_env env, napi_value value, uint32_t* result);
napi_status napi_get_value_int32(napi_env env, napi_value value, int32_t* result);
napi_status napi_create_string_utf8(napi_env env, const char* str, size_t length, napi_value* result);
napi_status napi_get_value_string_utf8(napi_env env, napi_value value, char* buf, size_t bufsize, size_t* result);
napi_status napi_create_arraybuffer(napi_env env, size_t byte_length, void** data, napi_value* result);
napi_status napi_create_typedarray(napi_env env, napi_typedarray_type type, size_t length, napi_value arraybuffer,
                                   size_t byte_offset, napi_value* result);
napi_status napi_create_object(napi_env env, napi_value* result);
napi_status napi_set_named_property(napi_env env, napi_value object, const char* utf8name, napi_value value);
napi_status napi_define_properties(napi_env env, napi_value object, size_t property_count,
                                   const napi_property_descriptor* properties);
#define NAPI_MODULE(modname, regfunc) napi_value textsift_module_init(napi_env e, napi_value x) { return regfunc(e, x); }
"""


def _strip_comments(src):
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.sub(r"//[^\n]*", "", src)


def test_napi_glue_type_checks_against_header(tmp_path):
    (tmp_path / "node_api.h").write_text(NODE_API_STUB)
    r = subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-fsyntax-only",
                        "-DNODE_GYP_MODULE_NAME=textsift_cuda", "-I", str(tmp_path), "-I", os.path.join(ROOT, "include"),
                        C_SRC], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_napi_glue_calls_only_declared_functions():
    header = _strip_comments(open(HEADER).read())
    declared = set(re.findall(r"\b(ts_(?:cuda|tok)_\w+)\s*\(", header))
    called = set(re.findall(r"\b(ts_(?:cuda|tok)_\w+)\s*\(", _strip_comments(open(C_SRC).read())))
    assert called and called <= declared, called - declared


def test_typescript_backend_matches_addon_exports():
    c = open(C_SRC).read()
    registered = set(re.findall(r'\{"(\w+)", NULL, \w+, NULL', c))
    ts = _strip_comments(open(TS_SRC).read())
    iface = ts[ts.index("export interface CudaApi"):]
    iface = iface[:iface.index("\n}")]
    declared = set(re.findall(r"^\s+(\w+)\(", iface, flags=re.M))
    assert declared == registered, (declared ^ registered)
    used = set(re.findall(r"\bthis\.api\.(\w+)\(", ts))
    assert used and used <= registered, used - registered
    # the InferenceBackend surface (browser/backends/abstract.ts:36-56)
    for member in ("readonly name", "async warmup()", "async forward(", "dispose()"):
        assert member in ts, member
