// qq3_addon.cc -- N-API addon exposing libqq3cuda.so (include/qq3.h) to the Node.js engines.
//
// This is the binding a QwenQwen3.js maintainer adds so that gguf.js, tokenizer.js and the
// engine forward()/generate() code stay in JavaScript while the arithmetic runs on a B200.
// It uses only the C N-API (node_api.h), so it builds against any Node >= 18 with
//   node-gyp rebuild        (binding.gyp in this folder)
// Node and its headers are not installed on the build machines of this repository, so this
// file is compiled only where a Node toolchain exists.
//
// Exported functions (all synchronous except forward/generate, which run on the libuv
// thread pool through napi_async_work so `await engine.forward(...)` keeps its meaning):
//   init(deviceIndex) -> ctx
//   uploadTensor(ctx, Uint8Array raw, ggmlType, shape[]) -> tensor
//   freeTensor(tensor)
//   modelCreate(ctx, desc) -> model          desc = {arch, nLayers, ..., layers:[{isAttn,isMoE,t:[19]}]}
//   forward(model, Int32Array tokens, seq, pos0, wantLogits, suppressId) -> Promise<{logits, argmax}>
//   generate(model, Int32Array prompt, maxSteps, thinkId, eosId, seq) -> Promise<Int32Array>
//   readRouting(model, moeLayer, recLen) -> Float32Array
//   setExpertMask(model, Int32Array) ; reset(model, seq) ; modelDestroy(model) ; destroy(ctx)
// Errors: a non-zero qq_* status becomes a thrown JS Error carrying qq_last_error().
#include <node_api.h>

#include <cstring>
#include <string>
#include <vector>

#include "qq3.h"  // include/ (built with -I include)

#define NAPI_CALL(env, call)                                        \
    do {                                                            \
        if ((call) != napi_ok) {                                    \
            napi_throw_error((env), nullptr, "N-API call failed");  \
            return nullptr;                                         \
        }                                                           \
    } while (0)

static napi_value throw_qq(napi_env env, int rc) {
    std::string msg = std::string("libqq3cuda: ") + qq_last_error() + " (" + std::to_string(rc) + ")";
    napi_throw_error(env, nullptr, msg.c_str());
    return nullptr;
}

static napi_value wrap_ptr(napi_env env, void* p) {
    napi_value v;
    napi_create_external(env, p, nullptr, nullptr, &v);
    return v;
}

static void* unwrap_ptr(napi_env env, napi_value v) {
    void* p = nullptr;
    napi_get_value_external(env, v, &p);
    return p;
}

static int32_t get_i32(napi_env env, napi_value v) {
    int32_t x = 0;
    napi_get_value_int32(env, v, &x);
    return x;
}

static double get_f64(napi_env env, napi_value v) {
    double x = 0;
    napi_get_value_double(env, v, &x);
    return x;
}

static napi_value prop(napi_env env, napi_value obj, const char* name) {
    napi_value v;
    napi_get_named_property(env, obj, name, &v);
    return v;
}

static bool is_null(napi_env env, napi_value v) {
    napi_valuetype t;
    napi_typeof(env, v, &t);
    return t == napi_null || t == napi_undefined;
}

template <class T>
static T* typed_data(napi_env env, napi_value arr, size_t* len) {
    napi_typedarray_type type;
    size_t length = 0, offset = 0;
    void* data = nullptr;
    napi_value ab;
    napi_get_typedarray_info(env, arr, &type, &length, &data, &ab, &offset);
    if (len) *len = length;
    return static_cast<T*>(data);
}

// init(deviceIndex) -> ctx
static napi_value Init(napi_env env, napi_callback_info info) {
    size_t argc = 1;
    napi_value argv[1];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    int dev = argc > 0 ? get_i32(env, argv[0]) : 0;
    qq_ctx* ctx = nullptr;
    int rc = qq_init(&dev, 1, &ctx);
    if (rc) return throw_qq(env, rc);
    return wrap_ptr(env, ctx);
}

// uploadTensor(ctx, Uint8Array raw, ggmlType, shape[]) -> tensor   (gguf.js meta -> device)
static napi_value UploadTensor(napi_env env, napi_callback_info info) {
    size_t argc = 4;
    napi_value argv[4];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    qq_ctx* ctx = static_cast<qq_ctx*>(unwrap_ptr(env, argv[0]));
    size_t n = 0;
    uint8_t* raw = typed_data<uint8_t>(env, argv[1], &n);
    int type = get_i32(env, argv[2]);
    uint32_t nd = 0;
    napi_get_array_length(env, argv[3], &nd);
    int64_t ne[4] = {1, 1, 1, 1};
    for (uint32_t i = 0; i < nd && i < 4; i++) {
        napi_value e;
        napi_get_element(env, argv[3], i, &e);
        ne[i] = (int64_t)get_f64(env, e);
    }
    qq_tensor* t = nullptr;
    int rc = qq_upload_tensor(ctx, raw, n, type, ne, (int)nd, &t);
    if (rc) return throw_qq(env, rc);
    return wrap_ptr(env, t);
}

static napi_value FreeTensor(napi_env env, napi_callback_info info) {
    size_t argc = 1;
    napi_value argv[1];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    int rc = qq_free_tensor(static_cast<qq_tensor*>(unwrap_ptr(env, argv[0])));
    if (rc) return throw_qq(env, rc);
    return nullptr;
}

// modelCreate(ctx, desc) -> model
static napi_value ModelCreate(napi_env env, napi_callback_info info) {
    size_t argc = 2;
    napi_value argv[2];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    qq_ctx* ctx = static_cast<qq_ctx*>(unwrap_ptr(env, argv[0]));
    napi_value d = argv[1];
    qq_model_desc desc;
    std::memset(&desc, 0, sizeof(desc));
    desc.arch = get_i32(env, prop(env, d, "arch"));
    desc.n_layers = get_i32(env, prop(env, d, "nLayers"));
    desc.n_embd = get_i32(env, prop(env, d, "nEmb"));
    desc.n_head = get_i32(env, prop(env, d, "nHeads"));
    desc.n_head_kv = get_i32(env, prop(env, d, "nHeadKV"));
    desc.head_dim = get_i32(env, prop(env, d, "headDim"));
    desc.n_vocab = get_i32(env, prop(env, d, "nVocab"));
    desc.n_expert = get_i32(env, prop(env, d, "nExperts"));
    desc.n_expert_used = get_i32(env, prop(env, d, "nExpertsUsed"));
    desc.max_ctx = get_i32(env, prop(env, d, "maxCtx"));
    desc.n_seq = get_i32(env, prop(env, d, "nSeq"));
    desc.rms_eps = (float)get_f64(env, prop(env, d, "eps"));
    desc.rope_base = get_f64(env, prop(env, d, "ropeFreqBase"));
    desc.tok_embd = static_cast<qq_tensor*>(unwrap_ptr(env, prop(env, d, "tokEmbd")));
    desc.output_norm = static_cast<qq_tensor*>(unwrap_ptr(env, prop(env, d, "outputNorm")));
    napi_value out = prop(env, d, "output");
    desc.output = is_null(env, out) ? nullptr : static_cast<qq_tensor*>(unwrap_ptr(env, out));
    std::vector<qq_layer_desc> layers(desc.n_layers);
    napi_value arr = prop(env, d, "layers");
    for (int l = 0; l < desc.n_layers; l++) {
        napi_value L;
        napi_get_element(env, arr, l, &L);
        layers[l].is_attn = get_i32(env, prop(env, L, "isAttn"));
        layers[l].is_moe = get_i32(env, prop(env, L, "isMoE"));
        napi_value ts = prop(env, L, "t");
        for (int s = 0; s < QQ_SLOT_COUNT; s++) {
            napi_value tv;
            napi_get_element(env, ts, s, &tv);
            layers[l].t[s] = is_null(env, tv) ? nullptr : static_cast<qq_tensor*>(unwrap_ptr(env, tv));
        }
    }
    desc.layers = layers.data();
    qq_model* m = nullptr;
    int rc = qq_model_create(ctx, &desc, &m);
    if (rc) return throw_qq(env, rc);
    return wrap_ptr(env, m);
}

// ---- forward as async work ----
struct ForwardWork {
    napi_async_work work;
    napi_deferred deferred;
    qq_model* m;
    std::vector<int32_t> tokens;
    int seq, pos0, want_logits, suppress, n_vocab;
    std::vector<float> logits;
    int32_t argmax = -1;
    int rc = 0;
    std::string err;
};

static void ForwardExecute(napi_env, void* data) {
    ForwardWork* w = static_cast<ForwardWork*>(data);
    if (w->want_logits) w->logits.resize(w->n_vocab);
    w->rc = qq_forward(w->m, w->tokens.data(), (int)w->tokens.size(), w->seq, w->pos0, w->want_logits,
                       w->want_logits ? w->logits.data() : nullptr, w->want_logits ? &w->argmax : nullptr, w->suppress);
    if (w->rc) w->err = qq_last_error();  // thread-local: read on the worker thread
}

static void ForwardComplete(napi_env env, napi_status, void* data) {
    ForwardWork* w = static_cast<ForwardWork*>(data);
    if (w->rc) {
        napi_value msg, err;
        napi_create_string_utf8(env, ("libqq3cuda: " + w->err).c_str(), NAPI_AUTO_LENGTH, &msg);
        napi_create_error(env, nullptr, msg, &err);
        napi_reject_deferred(env, w->deferred, err);
    } else {
        napi_value result, am;
        napi_create_object(env, &result);
        napi_create_int32(env, w->argmax, &am);
        napi_set_named_property(env, result, "argmax", am);
        if (w->want_logits) {
            napi_value ab, f32;
            void* buf = nullptr;
            napi_create_arraybuffer(env, w->logits.size() * 4, &buf, &ab);
            std::memcpy(buf, w->logits.data(), w->logits.size() * 4);
            napi_create_typedarray(env, napi_float32_array, w->logits.size(), ab, 0, &f32);
            napi_set_named_property(env, result, "logits", f32);
        }
        napi_resolve_deferred(env, w->deferred, result);
    }
    napi_delete_async_work(env, w->work);
    delete w;
}

// forward(model, Int32Array tokens, seq, pos0, wantLogits, suppressId, nVocab) -> Promise
static napi_value Forward(napi_env env, napi_callback_info info) {
    size_t argc = 7;
    napi_value argv[7];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    ForwardWork* w = new ForwardWork;
    w->m = static_cast<qq_model*>(unwrap_ptr(env, argv[0]));
    size_t n = 0;
    int32_t* t = typed_data<int32_t>(env, argv[1], &n);
    w->tokens.assign(t, t + n);
    w->seq = get_i32(env, argv[2]);
    w->pos0 = get_i32(env, argv[3]);
    w->want_logits = get_i32(env, argv[4]);
    w->suppress = get_i32(env, argv[5]);
    w->n_vocab = get_i32(env, argv[6]);
    napi_value promise, name;
    napi_create_promise(env, &w->deferred, &promise);
    napi_create_string_utf8(env, "qq3.forward", NAPI_AUTO_LENGTH, &name);
    napi_create_async_work(env, nullptr, name, ForwardExecute, ForwardComplete, w, &w->work);
    napi_queue_async_work(env, w->work);
    return promise;
}

// ---- forwardBatch: one step of several sequences (qq_forward_batch) as async work ----
struct BatchWork {
    napi_async_work work;
    napi_deferred deferred;
    qq_model* m;
    std::vector<int32_t> seqs, tokens, positions, argmax;
    int want_logits, suppress, n_vocab;
    std::vector<float> logits;
    int rc = 0;
    std::string err;
};

static void BatchExecute(napi_env, void* data) {
    BatchWork* w = static_cast<BatchWork*>(data);
    const int n = (int)w->seqs.size();
    if (w->want_logits) {
        w->logits.resize((size_t)n * w->n_vocab);
        w->argmax.assign(n, -1);
    }
    w->rc = qq_forward_batch(w->m, w->seqs.data(), w->tokens.data(), w->positions.data(), n, w->want_logits,
                             w->want_logits ? w->logits.data() : nullptr, w->want_logits ? w->argmax.data() : nullptr,
                             w->suppress);
    if (w->rc) w->err = qq_last_error();
}

static void BatchComplete(napi_env env, napi_status, void* data) {
    BatchWork* w = static_cast<BatchWork*>(data);
    if (w->rc) {
        napi_value msg, err;
        napi_create_string_utf8(env, ("libqq3cuda: " + w->err).c_str(), NAPI_AUTO_LENGTH, &msg);
        napi_create_error(env, nullptr, msg, &err);
        napi_reject_deferred(env, w->deferred, err);
    } else {
        napi_value result;
        napi_create_object(env, &result);
        if (w->want_logits) {
            napi_value ab, f32, ab2, i32;
            void* buf = nullptr;
            napi_create_arraybuffer(env, w->logits.size() * 4, &buf, &ab);
            std::memcpy(buf, w->logits.data(), w->logits.size() * 4);
            napi_create_typedarray(env, napi_float32_array, w->logits.size(), ab, 0, &f32);
            napi_set_named_property(env, result, "logits", f32);  // row i = sequence seqs[i]
            napi_create_arraybuffer(env, w->argmax.size() * 4, &buf, &ab2);
            std::memcpy(buf, w->argmax.data(), w->argmax.size() * 4);
            napi_create_typedarray(env, napi_int32_array, w->argmax.size(), ab2, 0, &i32);
            napi_set_named_property(env, result, "argmax", i32);
        }
        napi_resolve_deferred(env, w->deferred, result);
    }
    napi_delete_async_work(env, w->work);
    delete w;
}

// forwardBatch(model, Int32Array seqs, Int32Array tokens, Int32Array positions, wantLogits, suppressId,
//              nVocab) -> Promise<{logits, argmax}>
static napi_value ForwardBatch(napi_env env, napi_callback_info info) {
    size_t argc = 7;
    napi_value argv[7];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    BatchWork* w = new BatchWork;
    w->m = static_cast<qq_model*>(unwrap_ptr(env, argv[0]));
    size_t n = 0;
    int32_t* p = typed_data<int32_t>(env, argv[1], &n);
    w->seqs.assign(p, p + n);
    p = typed_data<int32_t>(env, argv[2], &n);
    w->tokens.assign(p, p + n);
    p = typed_data<int32_t>(env, argv[3], &n);
    w->positions.assign(p, p + n);
    w->want_logits = get_i32(env, argv[4]);
    w->suppress = get_i32(env, argv[5]);
    w->n_vocab = get_i32(env, argv[6]);
    napi_value promise, name;
    napi_create_promise(env, &w->deferred, &promise);
    napi_create_string_utf8(env, "qq3.forwardBatch", NAPI_AUTO_LENGTH, &name);
    napi_create_async_work(env, nullptr, name, BatchExecute, BatchComplete, w, &w->work);
    napi_queue_async_work(env, w->work);
    return promise;
}

// readRouting(model, moeLayer, recLen) -> Float32Array [idx | w | probs] (webgpu.js:1617-1618)
static napi_value ReadRouting(napi_env env, napi_callback_info info) {
    size_t argc = 3;
    napi_value argv[3];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    qq_model* m = static_cast<qq_model*>(unwrap_ptr(env, argv[0]));
    int layer = get_i32(env, argv[1]), len = get_i32(env, argv[2]);
    napi_value ab, f32;
    void* buf = nullptr;
    napi_create_arraybuffer(env, (size_t)len * 4, &buf, &ab);
    int rc = qq_read_routing(m, layer, static_cast<float*>(buf));
    if (rc) return throw_qq(env, rc);
    napi_create_typedarray(env, napi_float32_array, len, ab, 0, &f32);
    return f32;
}

static napi_value SetExpertMask(napi_env env, napi_callback_info info) {
    size_t argc = 2;
    napi_value argv[2];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    size_t n = 0;
    int32_t* ids = typed_data<int32_t>(env, argv[1], &n);
    int rc = qq_set_expert_mask(static_cast<qq_model*>(unwrap_ptr(env, argv[0])), ids, (int)n);
    if (rc) return throw_qq(env, rc);
    return nullptr;
}

static napi_value Reset(napi_env env, napi_callback_info info) {
    size_t argc = 2;
    napi_value argv[2];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    int rc = qq_reset(static_cast<qq_model*>(unwrap_ptr(env, argv[0])), argc > 1 ? get_i32(env, argv[1]) : 0);
    if (rc) return throw_qq(env, rc);
    return nullptr;
}

static napi_value ModelDestroy(napi_env env, napi_callback_info info) {
    size_t argc = 1;
    napi_value argv[1];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    int rc = qq_model_destroy(static_cast<qq_model*>(unwrap_ptr(env, argv[0])));
    if (rc) return throw_qq(env, rc);
    return nullptr;
}

static napi_value Destroy(napi_env env, napi_callback_info info) {
    size_t argc = 1;
    napi_value argv[1];
    NAPI_CALL(env, napi_get_cb_info(env, info, &argc, argv, nullptr, nullptr));
    int rc = qq_destroy(static_cast<qq_ctx*>(unwrap_ptr(env, argv[0])));
    if (rc) return throw_qq(env, rc);
    return nullptr;
}

static napi_value ModuleInit(napi_env env, napi_value exports) {
    napi_property_descriptor props[] = {
        {"init", nullptr, Init, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"uploadTensor", nullptr, UploadTensor, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"freeTensor", nullptr, FreeTensor, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"modelCreate", nullptr, ModelCreate, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"forward", nullptr, Forward, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"forwardBatch", nullptr, ForwardBatch, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"readRouting", nullptr, ReadRouting, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"setExpertMask", nullptr, SetExpertMask, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"reset", nullptr, Reset, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"modelDestroy", nullptr, ModelDestroy, nullptr, nullptr, nullptr, napi_default, nullptr},
        {"destroy", nullptr, Destroy, nullptr, nullptr, nullptr, napi_default, nullptr},
    };
    napi_define_properties(env, exports, sizeof(props) / sizeof(props[0]), props);
    return exports;
}

NAPI_MODULE(NODE_GYP_MODULE_NAME, ModuleInit)
