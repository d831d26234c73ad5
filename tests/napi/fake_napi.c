/*
 * A stand-in for the Node-API runtime - TEST INFRASTRUCTURE ONLY.  No Node.js exists in
 * this image or on the GPU box; this implements the Node-API functions the addon uses
 * (tests/napi/node_api.h) over a small value model (numbers, booleans, null, objects,
 * arrays, typed arrays over caller-owned buffers, externals with finalizers, functions)
 * and a pending-exception slot per environment, so tests can call the addon's exported
 * functions the way JavaScript would and read back results and thrown errors.  Values are
 * never freed (a test process is short-lived); fake_gc() runs the externals' finalizers.
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "node_api.h"

enum kind { K_UNDEF, K_NULL, K_BOOL, K_NUM, K_OBJ, K_EXT, K_TYPED, K_ARRAY, K_FUNC, K_ABUF };
enum { MAX_PROPS = 64 };

struct napi_value__ {
    enum kind k;
    double num;
    bool b;
    /* external */
    void *ext;
    napi_finalize fin;
    void *hint;
    bool finalized;
    /* typed array / array buffer */
    napi_typedarray_type ttype;
    size_t len;
    void *data;
    /* object */
    int nprops;
    char *pname[MAX_PROPS];
    napi_value pval[MAX_PROPS];
    /* array */
    size_t alen;
    napi_value *elems;
    /* function */
    napi_callback fn;
    void *fndata;
};

struct napi_env__ {
    int pending;   /* 0 none, 1 Error, 2 RangeError */
    char msg[1024];
};

struct napi_callback_info__ {
    size_t argc;
    napi_value *argv;
    void *data;
};

static napi_value externals[4096];
static int n_externals;

static napi_value new_value(enum kind k) {
    napi_value v = (napi_value)calloc(1, sizeof(struct napi_value__));
    v->k = k;
    return v;
}

static size_t elem_size(napi_typedarray_type t) {
    switch (t) {
        case napi_int8_array:
        case napi_uint8_array:
        case napi_uint8_clamped_array: return 1;
        case napi_int16_array:
        case napi_uint16_array: return 2;
        case napi_int32_array:
        case napi_uint32_array:
        case napi_float32_array: return 4;
        default: return 8;
    }
}

/* ---- the Node-API functions ---- */

napi_status napi_get_cb_info(napi_env env, napi_callback_info cbinfo, size_t *argc, napi_value *argv,
                             napi_value *this_arg, void **data) {
    (void)env;
    if (argv && argc)
        for (size_t i = 0; i < *argc; ++i) argv[i] = i < cbinfo->argc ? cbinfo->argv[i] : new_value(K_UNDEF);
    if (argc) *argc = cbinfo->argc;
    if (this_arg) *this_arg = new_value(K_UNDEF);
    if (data) *data = cbinfo->data;
    return napi_ok;
}

napi_status napi_typeof(napi_env env, napi_value value, napi_valuetype *result) {
    (void)env;
    switch (value->k) {
        case K_UNDEF: *result = napi_undefined; break;
        case K_NULL: *result = napi_null; break;
        case K_BOOL: *result = napi_boolean; break;
        case K_NUM: *result = napi_number; break;
        case K_EXT: *result = napi_external; break;
        case K_FUNC: *result = napi_function; break;
        default: *result = napi_object; break;
    }
    return napi_ok;
}

napi_status napi_get_value_uint32(napi_env env, napi_value value, uint32_t *result) {
    (void)env;
    if (value->k != K_NUM) return napi_number_expected;
    *result = (uint32_t)value->num;
    return napi_ok;
}

napi_status napi_get_value_bool(napi_env env, napi_value value, bool *result) {
    (void)env;
    if (value->k != K_BOOL) return napi_boolean_expected;
    *result = value->b;
    return napi_ok;
}

napi_status napi_is_typedarray(napi_env env, napi_value value, bool *result) {
    (void)env;
    *result = value->k == K_TYPED;
    return napi_ok;
}

napi_status napi_get_typedarray_info(napi_env env, napi_value v, napi_typedarray_type *type, size_t *length,
                                     void **data, napi_value *arraybuffer, size_t *byte_offset) {
    (void)env;
    if (v->k != K_TYPED) return napi_invalid_arg;
    if (type) *type = v->ttype;
    if (length) *length = v->len;
    if (data) *data = v->data;
    if (arraybuffer) *arraybuffer = NULL;
    if (byte_offset) *byte_offset = 0;
    return napi_ok;
}

napi_status napi_create_arraybuffer(napi_env env, size_t byte_length, void **data, napi_value *result) {
    (void)env;
    napi_value v = new_value(K_ABUF);
    v->data = calloc(byte_length ? byte_length : 1, 1);
    v->len = byte_length;
    if (data) *data = v->data;
    *result = v;
    return napi_ok;
}

napi_status napi_create_typedarray(napi_env env, napi_typedarray_type type, size_t length, napi_value arraybuffer,
                                   size_t byte_offset, napi_value *result) {
    (void)env;
    if (!arraybuffer || arraybuffer->k != K_ABUF || byte_offset + length * elem_size(type) > arraybuffer->len)
        return napi_invalid_arg;
    napi_value v = new_value(K_TYPED);
    v->ttype = type;
    v->len = length;
    v->data = (char *)arraybuffer->data + byte_offset;
    *result = v;
    return napi_ok;
}

napi_status napi_create_external(napi_env env, void *data, napi_finalize finalize_cb, void *finalize_hint,
                                 napi_value *result) {
    (void)env;
    napi_value v = new_value(K_EXT);
    v->ext = data;
    v->fin = finalize_cb;
    v->hint = finalize_hint;
    if (n_externals < (int)(sizeof externals / sizeof externals[0])) externals[n_externals++] = v;
    *result = v;
    return napi_ok;
}

napi_status napi_get_value_external(napi_env env, napi_value value, void **result) {
    (void)env;
    if (value->k != K_EXT) return napi_invalid_arg;
    *result = value->ext;
    return napi_ok;
}

napi_status napi_create_object(napi_env env, napi_value *result) {
    (void)env;
    *result = new_value(K_OBJ);
    return napi_ok;
}

napi_status napi_set_named_property(napi_env env, napi_value object, const char *name, napi_value value) {
    (void)env;
    if (object->k != K_OBJ || object->nprops >= MAX_PROPS) return napi_object_expected;
    for (int i = 0; i < object->nprops; ++i)
        if (!strcmp(object->pname[i], name)) {
            object->pval[i] = value;
            return napi_ok;
        }
    const size_t n = strlen(name) + 1;
    object->pname[object->nprops] = (char *)memcpy(malloc(n), name, n);
    object->pval[object->nprops++] = value;
    return napi_ok;
}

napi_status napi_create_uint32(napi_env env, uint32_t value, napi_value *result) {
    (void)env;
    napi_value v = new_value(K_NUM);
    v->num = value;
    *result = v;
    return napi_ok;
}

napi_status napi_get_array_length(napi_env env, napi_value value, uint32_t *result) {
    (void)env;
    if (value->k != K_ARRAY) return napi_array_expected;
    *result = (uint32_t)value->alen;
    return napi_ok;
}

napi_status napi_get_element(napi_env env, napi_value object, uint32_t index, napi_value *result) {
    (void)env;
    if (object->k != K_ARRAY) return napi_array_expected;
    *result = index < object->alen ? object->elems[index] : new_value(K_UNDEF);
    return napi_ok;
}

napi_status napi_create_function(napi_env env, const char *utf8name, size_t length, napi_callback cb, void *data,
                                 napi_value *result) {
    (void)env;
    (void)utf8name;
    (void)length;
    napi_value v = new_value(K_FUNC);
    v->fn = cb;
    v->fndata = data;
    *result = v;
    return napi_ok;
}

static napi_status throw_kind(napi_env env, int kind, const char *msg) {
    if (env->pending) return napi_pending_exception;
    env->pending = kind;
    snprintf(env->msg, sizeof env->msg, "%s", msg ? msg : "");
    return napi_ok;
}

napi_status napi_throw_error(napi_env env, const char *code, const char *msg) {
    (void)code;
    return throw_kind(env, 1, msg);
}

napi_status napi_throw_range_error(napi_env env, const char *code, const char *msg) {
    (void)code;
    return throw_kind(env, 2, msg);
}

/* ---- the test harness's side (called through ctypes) ---- */

napi_value bgtq_napi_init(napi_env env, napi_value exports);

napi_env fake_env(void) { return (napi_env)calloc(1, sizeof(struct napi_env__)); }

napi_value fake_module(napi_env env) {
    napi_value exports = new_value(K_OBJ);
    return bgtq_napi_init(env, exports);
}

napi_value fake_undefined(void) { return new_value(K_UNDEF); }
napi_value fake_null(void) { return new_value(K_NULL); }
napi_value fake_bool(int b) {
    napi_value v = new_value(K_BOOL);
    v->b = b != 0;
    return v;
}
napi_value fake_number(double x) {
    napi_value v = new_value(K_NUM);
    v->num = x;
    return v;
}
/* a typed array over the caller's buffer (not copied: the caller keeps it alive) */
napi_value fake_typed(int type, void *data, size_t length) {
    napi_value v = new_value(K_TYPED);
    v->ttype = (napi_typedarray_type)type;
    v->len = length;
    v->data = data;
    return v;
}
napi_value fake_array(napi_value *elems, size_t n) {
    napi_value v = new_value(K_ARRAY);
    v->alen = n;
    v->elems = (napi_value *)calloc(n ? n : 1, sizeof(napi_value));
    for (size_t i = 0; i < n; ++i) v->elems[i] = elems[i];
    return v;
}

/* call exports[name](argv...): NULL result means undefined; check fake_exception after */
napi_value fake_call(napi_env env, napi_value exports, const char *name, napi_value *argv, size_t argc) {
    for (int i = 0; i < exports->nprops; ++i)
        if (!strcmp(exports->pname[i], name) && exports->pval[i]->k == K_FUNC) {
            struct napi_callback_info__ info = {argc, argv, exports->pval[i]->fndata};
            napi_value r = exports->pval[i]->fn(env, &info);
            return r ? r : new_value(K_UNDEF);
        }
    throw_kind(env, 1, "not a function");
    return new_value(K_UNDEF);
}

/* 0: no exception; 1: Error; 2: RangeError (message copied, exception cleared) */
int fake_exception(napi_env env, char *msg, size_t cap) {
    const int k = env->pending;
    if (k && msg && cap) snprintf(msg, cap, "%s", env->msg);
    env->pending = 0;
    env->msg[0] = 0;
    return k;
}

int fake_kind(napi_value v) { return (int)v->k; }
double fake_get_number(napi_value v) { return v->k == K_NUM ? v->num : -1.0; }
napi_value fake_get(napi_value obj, const char *name) {
    if (obj->k == K_OBJ)
        for (int i = 0; i < obj->nprops; ++i)
            if (!strcmp(obj->pname[i], name)) return obj->pval[i];
    return new_value(K_UNDEF);
}
/* a typed array's element type, length and data pointer */
int fake_typed_info(napi_value v, void **data, size_t *length) {
    if (v->k != K_TYPED) return -1;
    *data = v->data;
    *length = v->len;
    return (int)v->ttype;
}

/* run the finalizers of every external not finalized yet (a garbage collection) */
int fake_gc(napi_env env) {
    int n = 0;
    for (int i = 0; i < n_externals; ++i)
        if (!externals[i]->finalized && externals[i]->fin) {
            externals[i]->fin(env, externals[i]->ext, externals[i]->hint);
            externals[i]->finalized = true;
            ++n;
        }
    return n;
}
