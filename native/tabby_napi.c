/*
 * tabby_napi.c -- zero-dependency N-API addon over libtabbysample.so.
 *
 * The boundary the reference's TypeScript host binds: src/engine/sampler.ts keeps its
 * surface (sample / sampleFromTopK / SeededRandom, sampler.ts:105-212) and calls these
 * functions instead of recording WGSL sampling dispatches (src/engine/forward.ts:520-601).
 * Status: not built in this repository's images (Node.js and its headers are absent); a
 * maintainer builds it with binding.gyp next to this file. tests/test_napi_source.py
 * checks on the CPU that every tabby_* call here matches include/tabby_sample.h.
 *
 * Exports
 *   create({device, maxTopK, maxRows, maxVocab}) -> handle (External)
 *   destroy(handle)
 *   sampleBatch(handle, logits: Float32Array, rows, vocab,
 *               params: Float64Array(3 * rows) [temperature, topK, topP per row],
 *               uniforms: Float64Array(rows)) -> {ids: Int32Array, outcomes: Float64Array}
 *       host buffers; tabby_sample_rows (copies inside, synchronous)
 *   sampleBatchAsync(...same...) -> Promise of the same, on a libuv worker thread
 *   sampleRowsDevice(handle, dLogits: BigInt, rowStride, rows, vocab, dParams: BigInt,
 *                    dUniforms: BigInt, dOut: BigInt, stream: BigInt)
 *       device pointers (e.g. from a CUDA-aware runtime); tabby_sample_rows_async
 *   sampleFromTopK(ids: Int32Array, logits: Float32Array, maxLogit, sumExp,
 *                  temperature, topP, u) -> outcome (Float64Array of 5)
 *       host float64 finalize (sampler.ts:147-212); tabby_sample_from_topk
 *   poolSize(temperature, topK, maxTopK) -> number (inference.worker.ts:120-123)
 *   abiVersion() -> number
 * Every failing call throws a JS Error carrying tabby_last_error(), as the reference
 * throws ForwardError / Error; nothing aborts.
 *
 * Outcome layout (Float64Array, 6 per row): id, probability, consideredCount, poolMass,
 * poolExhausted (0/1), status.
 */
#include <node_api.h>
#include <stdlib.h>
#include <string.h>

#include "tabby_sample.h"

#define OUT_FIELDS 6

static napi_value throw_last(napi_env env) {
  napi_throw_error(env, NULL, tabby_last_error());
  return NULL;
}

static napi_value throw_msg(napi_env env, const char *msg) {
  napi_throw_error(env, NULL, msg);
  return NULL;
}

static int32_t get_i32(napi_env env, napi_value obj, const char *name, int32_t dflt) {
  napi_value v;
  bool has = false;
  int32_t out = dflt;
  if (napi_has_named_property(env, obj, name, &has) == napi_ok && has &&
      napi_get_named_property(env, obj, name, &v) == napi_ok)
    napi_get_value_int32(env, v, &out);
  return out;
}

static void *get_ptr(napi_env env, napi_value v) {
  uint64_t x = 0;
  bool lossless = false;
  napi_get_value_bigint_uint64(env, v, &x, &lossless);
  return (void *)(uintptr_t)x;
}

static void finalize_handle(napi_env env, void *data, void *hint) {
  (void)env;
  (void)hint;
  if (data) tabby_sampler_destroy((tabby_sampler *)data);
}

static tabby_sampler *get_handle(napi_env env, napi_value v) {
  void *p = NULL;
  napi_get_value_external(env, v, &p);
  return (tabby_sampler *)p;
}

static napi_value Create(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1], ext;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  tabby_sampler_config c;
  memset(&c, 0, sizeof(c));
  if (argc >= 1) {
    c.device = get_i32(env, argv[0], "device", 0);
    c.max_top_k = get_i32(env, argv[0], "maxTopK", 0);
    c.max_rows = get_i32(env, argv[0], "maxRows", 0);
    c.max_vocab = get_i32(env, argv[0], "maxVocab", 0);
  }
  tabby_sampler *s = NULL;
  if (tabby_sampler_create(&c, &s) != TABBY_OK) return throw_last(env);
  napi_create_external(env, s, finalize_handle, NULL, &ext);
  return ext;
}

static napi_value Destroy(napi_env env, napi_callback_info info) {
  size_t argc = 1;
  napi_value argv[1];
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  /* The External's finalizer frees the handle; destroy() only checks the argument. */
  if (argc < 1 || !get_handle(env, argv[0])) return throw_msg(env, "destroy: no handle");
  return NULL;
}

/* The arguments of one batch call, read on the JS thread. */
typedef struct {
  tabby_sampler *s;
  const float *logits;
  int32_t rows, vocab;
  tabby_sampling_params *params;
  const double *uniforms;
  tabby_sample_outcome *out;
  int status;
  char error[256];
  napi_ref refs[3]; /* keep the typed arrays alive during async work */
  napi_deferred deferred;
  napi_async_work work;
} Batch;

static int read_batch(napi_env env, napi_value *argv, size_t argc, Batch *b) {
  if (argc < 6) return 0;
  size_t n_logits = 0, n_params = 0, n_u = 0;
  void *lg = NULL, *pp = NULL, *uu = NULL;
  b->s = get_handle(env, argv[0]);
  napi_get_typedarray_info(env, argv[1], NULL, &n_logits, &lg, NULL, NULL);
  napi_get_value_int32(env, argv[2], &b->rows);
  napi_get_value_int32(env, argv[3], &b->vocab);
  napi_get_typedarray_info(env, argv[4], NULL, &n_params, &pp, NULL, NULL);
  napi_get_typedarray_info(env, argv[5], NULL, &n_u, &uu, NULL, NULL);
  if (!b->s || b->rows < 0 || b->vocab < 1 || n_logits < (size_t)b->rows * b->vocab ||
      n_params < 3 * (size_t)b->rows || n_u < (size_t)b->rows)
    return 0;
  b->logits = (const float *)lg;
  b->uniforms = (const double *)uu;
  const double *p = (const double *)pp;
  b->params = (tabby_sampling_params *)calloc((size_t)b->rows + 1, sizeof(tabby_sampling_params));
  b->out = (tabby_sample_outcome *)calloc((size_t)b->rows + 1, sizeof(tabby_sample_outcome));
  for (int32_t r = 0; r < b->rows; r++) {
    b->params[r].temperature = p[3 * r];
    b->params[r].top_k = (int32_t)p[3 * r + 1];
    b->params[r].top_p = p[3 * r + 2];
  }
  return 1;
}

static void run_batch(Batch *b) {
  b->status = tabby_sample_rows(b->s, b->logits, b->vocab, b->rows, b->vocab, b->params,
                                b->uniforms, b->out, NULL, NULL, 0);
  if (b->status != TABBY_OK) strncpy(b->error, tabby_last_error(), sizeof(b->error) - 1);
}

static napi_value batch_result(napi_env env, const Batch *b) {
  napi_value res, ids_buf, ids, oc_buf, oc;
  int32_t *ids_data = NULL;
  double *oc_data = NULL;
  napi_create_arraybuffer(env, 4 * (size_t)b->rows, (void **)&ids_data, &ids_buf);
  napi_create_arraybuffer(env, 8 * OUT_FIELDS * (size_t)b->rows, (void **)&oc_data, &oc_buf);
  for (int32_t r = 0; r < b->rows; r++) {
    const tabby_sample_outcome *o = &b->out[r];
    ids_data[r] = o->id;
    oc_data[OUT_FIELDS * r + 0] = o->id;
    oc_data[OUT_FIELDS * r + 1] = o->probability;
    oc_data[OUT_FIELDS * r + 2] = o->considered_count;
    oc_data[OUT_FIELDS * r + 3] = o->pool_mass;
    oc_data[OUT_FIELDS * r + 4] = o->pool_exhausted;
    oc_data[OUT_FIELDS * r + 5] = o->status;
  }
  napi_create_typedarray(env, napi_int32_array, (size_t)b->rows, ids_buf, 0, &ids);
  napi_create_typedarray(env, napi_float64_array, OUT_FIELDS * (size_t)b->rows, oc_buf, 0, &oc);
  napi_create_object(env, &res);
  napi_set_named_property(env, res, "ids", ids);
  napi_set_named_property(env, res, "outcomes", oc);
  return res;
}

static void free_batch(Batch *b) {
  free(b->params);
  free(b->out);
}

static napi_value SampleBatch(napi_env env, napi_callback_info info) {
  size_t argc = 6;
  napi_value argv[6];
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Batch b;
  memset(&b, 0, sizeof(b));
  if (!read_batch(env, argv, argc, &b)) return throw_msg(env, "sampleBatch: bad arguments");
  run_batch(&b);
  if (b.status != TABBY_OK) {
    free_batch(&b);
    return throw_msg(env, b.error);
  }
  napi_value res = batch_result(env, &b);
  free_batch(&b);
  return res;
}

static void async_execute(napi_env env, void *data) {
  (void)env;
  run_batch((Batch *)data);
}

static void async_complete(napi_env env, napi_status status, void *data) {
  Batch *b = (Batch *)data;
  if (status == napi_ok && b->status == TABBY_OK) {
    napi_resolve_deferred(env, b->deferred, batch_result(env, b));
  } else {
    napi_value msg, err;
    napi_create_string_utf8(env, b->status != TABBY_OK ? b->error : "sampleBatchAsync failed",
                            NAPI_AUTO_LENGTH, &msg);
    napi_create_error(env, NULL, msg, &err);
    napi_reject_deferred(env, b->deferred, err);
  }
  for (int i = 0; i < 3; i++) napi_delete_reference(env, b->refs[i]);
  napi_delete_async_work(env, b->work);
  free_batch(b);
  free(b);
}

static napi_value SampleBatchAsync(napi_env env, napi_callback_info info) {
  size_t argc = 6;
  napi_value argv[6], promise, name;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  Batch *b = (Batch *)calloc(1, sizeof(Batch));
  if (!b || !read_batch(env, argv, argc, b)) {
    if (b) free(b);
    return throw_msg(env, "sampleBatchAsync: bad arguments");
  }
  napi_create_reference(env, argv[1], 1, &b->refs[0]);
  napi_create_reference(env, argv[4], 1, &b->refs[1]);
  napi_create_reference(env, argv[5], 1, &b->refs[2]);
  napi_create_promise(env, &b->deferred, &promise);
  napi_create_string_utf8(env, "tabby.sampleBatch", NAPI_AUTO_LENGTH, &name);
  napi_create_async_work(env, NULL, name, async_execute, async_complete, b, &b->work);
  napi_queue_async_work(env, b->work);
  return promise;
}

static napi_value SampleRowsDevice(napi_env env, napi_callback_info info) {
  size_t argc = 9;
  napi_value argv[9];
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  if (argc < 9) return throw_msg(env, "sampleRowsDevice: 9 arguments expected");
  int64_t stride = 0;
  int32_t rows = 0, vocab = 0;
  napi_get_value_int64(env, argv[2], &stride);
  napi_get_value_int32(env, argv[3], &rows);
  napi_get_value_int32(env, argv[4], &vocab);
  const int st = tabby_sample_rows_async(
      get_handle(env, argv[0]), (const float *)get_ptr(env, argv[1]), stride, rows, vocab,
      (const tabby_sampling_params *)get_ptr(env, argv[5]), (const double *)get_ptr(env, argv[6]),
      (tabby_sample_outcome *)get_ptr(env, argv[7]), NULL, NULL, 0, get_ptr(env, argv[8]));
  if (st != TABBY_OK) return throw_last(env);
  return NULL;
}

static napi_value SampleFromTopK(napi_env env, napi_callback_info info) {
  size_t argc = 7;
  napi_value argv[7], res, buf;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  if (argc < 7) return throw_msg(env, "sampleFromTopK: 7 arguments expected");
  size_t n_ids = 0, n_logits = 0;
  void *ids = NULL, *lg = NULL;
  double max_logit, sum_exp, u;
  tabby_sampling_params p;
  memset(&p, 0, sizeof(p));
  napi_get_typedarray_info(env, argv[0], NULL, &n_ids, &ids, NULL, NULL);
  napi_get_typedarray_info(env, argv[1], NULL, &n_logits, &lg, NULL, NULL);
  napi_get_value_double(env, argv[2], &max_logit);
  napi_get_value_double(env, argv[3], &sum_exp);
  napi_get_value_double(env, argv[4], &p.temperature);
  napi_get_value_double(env, argv[5], &p.top_p);
  napi_get_value_double(env, argv[6], &u);
  if (n_ids != n_logits) return throw_msg(env, "sampleFromTopK: ids and logits differ in length");
  tabby_sample_outcome o;
  if (tabby_sample_from_topk((const int32_t *)ids, (const float *)lg, (int32_t)n_ids,
                             (float)max_logit, (float)sum_exp, &p, u, &o) != TABBY_OK)
    return throw_last(env);
  double *d = NULL;
  napi_create_arraybuffer(env, 8 * 5, (void **)&d, &buf);
  d[0] = o.id;
  d[1] = o.probability;
  d[2] = o.considered_count;
  d[3] = o.pool_mass;
  d[4] = o.pool_exhausted;
  napi_create_typedarray(env, napi_float64_array, 5, buf, 0, &res);
  return res;
}

static napi_value PoolSize(napi_env env, napi_callback_info info) {
  size_t argc = 3;
  napi_value argv[3], res;
  napi_get_cb_info(env, info, &argc, argv, NULL, NULL);
  double t = 0;
  int32_t k = 0, cap = TABBY_DEFAULT_MAX_TOP_K;
  if (argc >= 1) napi_get_value_double(env, argv[0], &t);
  if (argc >= 2) napi_get_value_int32(env, argv[1], &k);
  if (argc >= 3) napi_get_value_int32(env, argv[2], &cap);
  napi_create_int32(env, tabby_pool_size(t, k, cap), &res);
  return res;
}

static napi_value AbiVersion(napi_env env, napi_callback_info info) {
  (void)info;
  napi_value res;
  napi_create_int32(env, tabby_abi_version(), &res);
  return res;
}

static void export_fn(napi_env env, napi_value exports, const char *name, napi_callback cb) {
  napi_value fn;
  napi_create_function(env, name, NAPI_AUTO_LENGTH, cb, NULL, &fn);
  napi_set_named_property(env, exports, name, fn);
}

NAPI_MODULE_INIT() {
  export_fn(env, exports, "create", Create);
  export_fn(env, exports, "destroy", Destroy);
  export_fn(env, exports, "sampleBatch", SampleBatch);
  export_fn(env, exports, "sampleBatchAsync", SampleBatchAsync);
  export_fn(env, exports, "sampleRowsDevice", SampleRowsDevice);
  export_fn(env, exports, "sampleFromTopK", SampleFromTopK);
  export_fn(env, exports, "poolSize", PoolSize);
  export_fn(env, exports, "abiVersion", AbiVersion);
  return exports;
}
