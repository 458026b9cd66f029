// C ABI of openmini_v1_b200 (include/openmini_b200.h).
//
// Every call marshals its C arguments into the Python engine
// (openmini_v1_b200.capi_backend) under the GIL and converts the answer back
// into C structs / buffers owned by the handle. A host without a Python
// interpreter gets one embedded by openmini_init(); inside a Python process
// the running interpreter is used.
#include <pybind11/embed.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/openmini_b200.h"

namespace py = pybind11;

struct openmini_model {
  int64_t handle;
};

struct openmini_context {
  int64_t handle;
  std::vector<float> logits;
};

namespace {

bool g_we_initialised = false;
openmini_log_callback_t g_log_cb = nullptr;
void* g_log_user = nullptr;

py::module_ backend() { return py::module_::import("openmini_v1_b200.capi_backend"); }

template <class F>
openmini_error_t guarded(F&& f, openmini_error_t on_error = OPENMINI_ERR_INFERENCE) {
  if (!Py_IsInitialized()) return OPENMINI_ERR_INVALID_PARAM;
  py::gil_scoped_acquire gil;
  try {
    return f();
  } catch (py::error_already_set& e) {
    const bool full = e.matches(PyExc_OverflowError);
    if (g_log_cb) g_log_cb(3, e.what(), g_log_user);
    return full ? OPENMINI_ERR_CONTEXT_FULL : on_error;
  } catch (std::exception& e) {
    if (g_log_cb) g_log_cb(3, e.what(), g_log_user);
    return on_error;
  }
}

void copy_str(char* dst, size_t n, const std::string& s) {
  std::strncpy(dst, s.c_str(), n - 1);
  dst[n - 1] = '\0';
}

}  // namespace

extern "C" {

openmini_error_t openmini_init(void) {
  if (!Py_IsInitialized()) {
    Py_InitializeEx(0);
    g_we_initialised = true;
    PyEval_SaveThread();  // release the GIL: every call re-acquires it
  }
  return guarded([] {
    backend();
    return OPENMINI_OK;
  });
}

void openmini_cleanup(void) {
  if (g_we_initialised && Py_IsInitialized()) {
    PyGILState_Ensure();
    Py_FinalizeEx();
    g_we_initialised = false;
  }
}

const char* openmini_version(void) { return OPENMINI_B200_VERSION; }

const char* const* openmini_get_backends(size_t* count) {
  static const char* const names[] = {"cuda-sm_100a", "cpu"};
  if (count) *count = 2;
  return names;
}

openmini_error_t openmini_load_model(const char* model_path, const openmini_config_t* config,
                                     openmini_model_t** out_model) {
  if (!model_path || !out_model) return OPENMINI_ERR_INVALID_PARAM;
  return guarded(
      [&] {
        const int n_ctx = config ? (int)config->n_ctx : 0;
        const int dev = config ? config->gpu_device_id : 0;
        const std::string q = config ? std::string(config->quant_type, strnlen(config->quant_type, 16)) : "";
        const int64_t h = backend().attr("load_model")(model_path, n_ctx, dev, q).cast<int64_t>();
        *out_model = new openmini_model{h};
        return OPENMINI_OK;
      },
      OPENMINI_ERR_MODEL_LOAD);
}

void openmini_free_model(openmini_model_t* model) {
  if (!model) return;
  guarded([&] {
    backend().attr("free_model")(model->handle);
    return OPENMINI_OK;
  });
  delete model;
}

openmini_error_t openmini_model_info(const openmini_model_t* model, openmini_model_info_t* info) {
  if (!model || !info) return OPENMINI_ERR_INVALID_PARAM;
  return guarded([&] {
    py::dict d = backend().attr("model_info")(model->handle);
    info->n_params = d["n_params"].cast<size_t>();
    info->n_layers = d["n_layers"].cast<size_t>();
    info->n_head = d["n_head"].cast<size_t>();
    info->n_head_kv = d["n_head_kv"].cast<size_t>();
    info->n_embd = d["n_embd"].cast<size_t>();
    info->n_vocab = d["n_vocab"].cast<size_t>();
    info->n_ff = d["n_ff"].cast<size_t>();
    copy_str(info->type, sizeof(info->type), d["type"].cast<std::string>());
    copy_str(info->quantization, sizeof(info->quantization), d["quantization"].cast<std::string>());
    return OPENMINI_OK;
  });
}

openmini_error_t openmini_new_context(const openmini_model_t* model, openmini_context_t** out_ctx) {
  if (!model || !out_ctx) return OPENMINI_ERR_INVALID_PARAM;
  return guarded(
      [&] {
        const int64_t h = backend().attr("new_context")(model->handle).cast<int64_t>();
        *out_ctx = new openmini_context{h, {}};
        return OPENMINI_OK;
      },
      OPENMINI_ERR_MEMORY);
}

void openmini_free_context(openmini_context_t* ctx) {
  if (!ctx) return;
  guarded([&] {
    backend().attr("free_context")(ctx->handle);
    return OPENMINI_OK;
  });
  delete ctx;
}

openmini_error_t openmini_reset_context(openmini_context_t* ctx) {
  if (!ctx) return OPENMINI_ERR_INVALID_PARAM;
  return guarded([&] {
    backend().attr("reset_context")(ctx->handle);
    ctx->logits.clear();
    return OPENMINI_OK;
  });
}

openmini_error_t openmini_generate(openmini_context_t* ctx, const char* prompt, int max_tokens, float temperature,
                                   float top_p, int top_k, openmini_result_t* result) {
  if (!ctx || !prompt || !result) return OPENMINI_ERR_INVALID_PARAM;
  return guarded([&] {
    py::dict d = backend().attr("generate")(ctx->handle, prompt, max_tokens, temperature, top_p, top_k);
    auto toks = d["tokens"].cast<std::vector<int>>();
    auto text = d["text"].cast<std::string>();
    std::memset(result, 0, sizeof(*result));
    result->tokens = static_cast<int*>(std::malloc(sizeof(int) * std::max<size_t>(toks.size(), 1)));
    result->text = static_cast<char*>(std::malloc(text.size() + 1));
    if (!result->tokens || !result->text) return OPENMINI_ERR_MEMORY;
    std::memcpy(result->tokens, toks.data(), sizeof(int) * toks.size());
    std::memcpy(result->text, text.c_str(), text.size() + 1);
    result->n_tokens = toks.size();
    result->prompt_tokens = d["prompt_tokens"].cast<uint64_t>();
    result->output_tokens = toks.size();
    result->prompt_processing_us = d["prompt_us"].cast<float>();
    result->token_generation_us = d["gen_us"].cast<float>();
    result->duration_us = (uint64_t)d["total_us"].cast<double>();
    result->tokens_per_second =
        result->token_generation_us > 0 ? toks.size() / (result->token_generation_us * 1e-6f) : 0.f;
    return OPENMINI_OK;
  });
}

openmini_error_t openmini_decode(openmini_context_t* ctx, const int* tokens, size_t n_tokens, bool preprocess_only) {
  if (!ctx || (!tokens && n_tokens)) return OPENMINI_ERR_INVALID_PARAM;
  return guarded([&] {
    std::vector<int> t(tokens, tokens + n_tokens);
    backend().attr("decode")(ctx->handle, t, preprocess_only);
    return OPENMINI_OK;
  });
}

int openmini_sample_token(openmini_context_t* ctx, float temperature, float top_p, int top_k) {
  if (!ctx) return -1;
  int tok = -1;
  const openmini_error_t e = guarded([&] {
    tok = backend().attr("sample_token")(ctx->handle, temperature, top_p, top_k).cast<int>();
    return OPENMINI_OK;
  });
  return e == OPENMINI_OK ? tok : -1;
}

openmini_error_t openmini_get_logits(openmini_context_t* ctx, float** logits, size_t* n_logits) {
  if (!ctx || !logits || !n_logits) return OPENMINI_ERR_INVALID_PARAM;
  return guarded([&] {
    py::object t = backend().attr("get_logits")(ctx->handle);
    if (t.is_none()) return OPENMINI_ERR_INFERENCE;
    auto v = t.attr("tolist")().cast<std::vector<float>>();
    ctx->logits = std::move(v);
    *logits = ctx->logits.data();
    *n_logits = ctx->logits.size();
    return OPENMINI_OK;
  });
}

void openmini_free_result(openmini_result_t* result) {
  if (!result) return;
  std::free(result->tokens);
  std::free(result->text);
  result->tokens = nullptr;
  result->text = nullptr;
  result->n_tokens = 0;
}

openmini_error_t openmini_get_stats(const openmini_context_t* ctx, openmini_stats_t* stats) {
  if (!ctx || !stats) return OPENMINI_ERR_INVALID_PARAM;
  return guarded([&] {
    py::dict d = backend().attr("stats")(ctx->handle);
    std::memset(stats, 0, sizeof(*stats));
    stats->total_prompt_us = d["total_prompt_us"].cast<uint64_t>();
    stats->total_gen_us = d["total_gen_us"].cast<uint64_t>();
    stats->total_tokens = d["total_tokens"].cast<uint64_t>();
    stats->tokens_per_second = d["tokens_per_second"].cast<float>();
    stats->gpu_memory_used_mb = d["gpu_memory_used_mb"].cast<float>();
    stats->n_prompt_tokens_processed = d["n_prompt_tokens_processed"].cast<size_t>();
    stats->n_tokens_generated = d["n_tokens_generated"].cast<size_t>();
    return OPENMINI_OK;
  });
}

void openmini_reset_stats(openmini_context_t* ctx) {
  if (!ctx) return;
  guarded([&] {
    backend().attr("reset_stats")(ctx->handle);
    return OPENMINI_OK;
  });
}

openmini_error_t openmini_set_log_callback(openmini_log_callback_t callback, void* user_data) {
  g_log_cb = callback;
  g_log_user = user_data;
  return guarded([&] {
    if (callback) {
      backend().attr("set_log")(py::cpp_function([](int level, std::string text) {
        if (g_log_cb) g_log_cb(level, text.c_str(), g_log_user);
      }));
    } else {
      backend().attr("set_log")(py::none());
    }
    return OPENMINI_OK;
  });
}

}  // extern "C"
