"""CPU: the N-API addon (native/tabby_napi.c) and the TypeScript wrapper (ts/sampler.ts)
agree with the C ABI they bind. Node.js is absent here, so the addon is compiled for a
syntax and type check against a stub of node_api.h (the N-API calls it makes, declared
with N-API's published signatures), and every tabby_* call is matched by name and
argument count against include/tabby_sample.h."""
import os
import re
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ADDON = os.path.join(ROOT, "native", "tabby_napi.c")
TS = os.path.join(ROOT, "ts", "sampler.ts")
HEADER = os.path.join(ROOT, "include", "tabby_sample.h")


def _split_args(s):
    depth, parts, cur = 0, [], ""
    for ch in s:
        if ch in "([{":
            depth += 1
        elif ch in ")]}":
            depth -= 1
        if ch == "," and depth == 0:
            parts.append(cur)
            cur = ""
        else:
            cur += ch
    if cur.strip():
        parts.append(cur)
    return parts


def _calls(src, prefix):
    """(name, argument count) of every call name(...) with the prefix."""
    out = []
    for m in re.finditer(r"\b(" + prefix + r"\w+)\s*\(", src):
        i, depth = m.end(), 1
        while depth:
            depth += {"(": 1, ")": -1}.get(src[i], 0)
            i += 1
        out.append((m.group(1), len(_split_args(src[m.end():i - 1]))))
    return out


def _declarations():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    decls = {}
    for m in re.finditer(r"TABBY_API\s+[\w\s\*]+?\b(tabby_\w+)\s*\(([^)]*)\)\s*;", src):
        args = m.group(2).strip()
        decls[m.group(1)] = 0 if args in ("", "void") else len(_split_args(args))
    return decls


def test_addon_calls_match_the_header():
    src = re.sub(r"/\*.*?\*/", "", open(ADDON).read(), flags=re.S)
    decls = _declarations()
    calls = _calls(src, "tabby_")
    assert calls, "the addon calls no tabby_* function"
    names = set()
    for name, n in calls:
        if name in ("tabby_napi",):
            continue
        assert name in decls, f"{name} is not declared in include/tabby_sample.h"
        assert n == decls[name], f"{name}: {n} arguments, the header declares {decls[name]}"
        names.add(name)
    for needed in ("tabby_sampler_create", "tabby_sample_rows", "tabby_sample_rows_async",
                   "tabby_sample_from_topk", "tabby_pool_size", "tabby_last_error"):
        assert needed in names


NODE_API_STUB = r"""
#include <stddef.h>
#include <stdint.h>
#include <stdbool.h>
typedef struct napi_env__ *napi_env;
typedef struct napi_value__ *napi_value;
typedef struct napi_ref__ *napi_ref;
typedef struct napi_deferred__ *napi_deferred;
typedef struct napi_async_work__ *napi_async_work;
typedef struct napi_callback_info__ *napi_callback_info;
typedef enum { napi_ok } napi_status;
typedef enum { napi_int32_array = 5, napi_float32_array = 7, napi_float64_array = 8 } napi_typedarray_type;
typedef napi_value (*napi_callback)(napi_env, napi_callback_info);
typedef void (*napi_finalize)(napi_env, void *, void *);
typedef void (*napi_async_execute_callback)(napi_env, void *);
typedef void (*napi_async_complete_callback)(napi_env, napi_status, void *);
#define NAPI_AUTO_LENGTH ((size_t)-1)
#define NAPI_MODULE_INIT() napi_value napi_register_module_v1(napi_env env, napi_value exports)
napi_status napi_get_cb_info(napi_env, napi_callback_info, size_t *, napi_value *, napi_value *, void **);
napi_status napi_throw_error(napi_env, const char *, const char *);
napi_status napi_has_named_property(napi_env, napi_value, const char *, bool *);
napi_status napi_get_named_property(napi_env, napi_value, const char *, napi_value *);
napi_status napi_set_named_property(napi_env, napi_value, const char *, napi_value);
napi_status napi_get_value_int32(napi_env, napi_value, int32_t *);
napi_status napi_get_value_int64(napi_env, napi_value, int64_t *);
napi_status napi_get_value_double(napi_env, napi_value, double *);
napi_status napi_get_value_bigint_uint64(napi_env, napi_value, uint64_t *, bool *);
napi_status napi_create_external(napi_env, void *, napi_finalize, void *, napi_value *);
napi_status napi_get_value_external(napi_env, napi_value, void **);
napi_status napi_get_typedarray_info(napi_env, napi_value, napi_typedarray_type *, size_t *, void **, napi_value *, size_t *);
napi_status napi_create_arraybuffer(napi_env, size_t, void **, napi_value *);
napi_status napi_create_typedarray(napi_env, napi_typedarray_type, size_t, napi_value, size_t, napi_value *);
napi_status napi_create_object(napi_env, napi_value *);
napi_status napi_create_int32(napi_env, int32_t, napi_value *);
napi_status napi_create_string_utf8(napi_env, const char *, size_t, napi_value *);
napi_status napi_create_error(napi_env, napi_value, napi_value, napi_value *);
napi_status napi_create_reference(napi_env, napi_value, uint32_t, napi_ref *);
napi_status napi_delete_reference(napi_env, napi_ref);
napi_status napi_create_promise(napi_env, napi_deferred *, napi_value *);
napi_status napi_resolve_deferred(napi_env, napi_deferred, napi_value);
napi_status napi_reject_deferred(napi_env, napi_deferred, napi_value);
napi_status napi_create_async_work(napi_env, napi_value, napi_value, napi_async_execute_callback, napi_async_complete_callback, void *, napi_async_work *);
napi_status napi_queue_async_work(napi_env, napi_async_work);
napi_status napi_delete_async_work(napi_env, napi_async_work);
napi_status napi_create_function(napi_env, const char *, size_t, napi_callback, void *, napi_value *);
"""


def test_addon_compiles_against_the_header(tmp_path):
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc absent")
    (tmp_path / "node_api.h").write_text(NODE_API_STUB)
    r = subprocess.run([gcc, "-std=c11", "-Wall", "-Werror", "-Wno-unused-parameter",
                        "-fsyntax-only", "-I", str(tmp_path), "-I",
                        os.path.join(ROOT, "include"), ADDON], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_typescript_uses_only_exported_addon_functions():
    exported = set(re.findall(r'export_fn\(env, exports, "(\w+)"', open(ADDON).read()))
    used = set(re.findall(r"\bnative\.(\w+)\(", open(TS).read()))
    assert used and used <= exported, used - exported
    ts = open(TS).read()
    # The reference's surface is kept.
    for name in ("export class SeededRandom", "export function sampleFromTopK",
                 "export interface SamplingParams", "export const DEFAULT_SAMPLING",
                 "sample(logits: Float32Array, params: SamplingParams, random: SeededRandom)"):
        assert name in ts, name
