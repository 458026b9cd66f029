/* C ABI of openmini_v1_b200 (exported by the native runtime library
 * openmini_v1_b200/_rt*.so).
 *
 * A C or C++ host loads a model, opens contexts (one token sequence each with
 * its own paged KV cache), and either generates text in one call or drives
 * the loop itself: decode (feed tokens) -> get_logits / sample_token -> decode.
 * The calls run the same engine, kernels and sampler as the Python API. The
 * library embeds CPython when the host has not initialised it; when called
 * from a Python process it attaches to the running interpreter.
 *
 * A host program without Python links libpython3 as well (the library
 * resolves the interpreter's symbols from the process).
 *
 * The function set, result codes and struct fields follow the reference's
 * llama.cpp-style header (openmini-server/native/include/openmini.h) so code
 * written against it ports by renaming the header.
 */
#pragma once
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define OPENMINI_API __attribute__((visibility("default")))
#else
#define OPENMINI_API
#endif

#define OPENMINI_B200_VERSION "0.1.0"

typedef struct openmini_context openmini_context_t;
typedef struct openmini_model openmini_model_t;

typedef enum {
  OPENMINI_OK = 0,
  OPENMINI_ERR_MEMORY = -1,
  OPENMINI_ERR_INVALID_PARAM = -2,
  OPENMINI_ERR_MODEL_LOAD = -3,
  OPENMINI_ERR_INFERENCE = -4,
  OPENMINI_ERR_UNSUPPORTED = -5,
  OPENMINI_ERR_CUDA = -6,
  OPENMINI_ERR_METAL = -7,
  OPENMINI_ERR_TOKENIZER = -8,
  OPENMINI_ERR_CONTEXT_FULL = -9,
} openmini_error_t;

typedef struct {
  uint32_t n_ctx;          /* max tokens per context (0: 4096) */
  uint32_t n_batch;
  uint32_t n_threads;
  int gpu_device_id;       /* -1: CPU */
  char quant_type[16];     /* "bf16" | "q4" | "int8" (weights re-packed for the GPU) */
  bool enable_kv_cache;
  bool enable_flash_attn;
  uint32_t kv_cache_size_mb;
  bool use_bitnet_lut;     /* accepted, unused */
  uint32_t lut_block_size; /* accepted, unused */
  float rope_scaling;
  float rope_freq_base;    /* 0: from the model file */
  float rope_freq_scale;
} openmini_config_t;

typedef struct {
  int* tokens;
  size_t n_tokens;
  char* text;
  uint64_t duration_us;
  uint64_t prompt_tokens;
  uint64_t output_tokens;
  float tokens_per_second;
  float prompt_processing_us;
  float token_generation_us;
} openmini_result_t;

typedef struct {
  size_t n_params;
  size_t n_layers;
  size_t n_head;
  size_t n_head_kv;
  size_t n_embd;
  size_t n_vocab;
  size_t n_ff;
  char type[64];
  char quantization[16];
} openmini_model_info_t;

typedef struct {
  uint64_t total_prompt_us;
  uint64_t total_gen_us;
  uint64_t total_tokens;
  float tokens_per_second;
  float memory_used_mb;
  float gpu_memory_used_mb;
  uint32_t cache_hit_rate;
  size_t n_prompt_tokens_processed;
  size_t n_tokens_generated;
} openmini_stats_t;

typedef void (*openmini_log_callback_t)(int level, const char* text, void* user_data);

OPENMINI_API openmini_error_t openmini_init(void);
OPENMINI_API void openmini_cleanup(void);
OPENMINI_API const char* openmini_version(void);
OPENMINI_API const char* const* openmini_get_backends(size_t* count);

/* model_path: a GGUF file, or "preset:<name>" for a random-init model of a named shape */
OPENMINI_API openmini_error_t openmini_load_model(const char* model_path, const openmini_config_t* config,
                                     openmini_model_t** out_model);
OPENMINI_API void openmini_free_model(openmini_model_t* model);
OPENMINI_API openmini_error_t openmini_model_info(const openmini_model_t* model, openmini_model_info_t* info);

OPENMINI_API openmini_error_t openmini_new_context(const openmini_model_t* model, openmini_context_t** out_ctx);
OPENMINI_API void openmini_free_context(openmini_context_t* ctx);
OPENMINI_API openmini_error_t openmini_reset_context(openmini_context_t* ctx);

OPENMINI_API openmini_error_t openmini_generate(openmini_context_t* ctx, const char* prompt, int max_tokens, float temperature,
                                   float top_p, int top_k, openmini_result_t* result);
OPENMINI_API openmini_error_t openmini_decode(openmini_context_t* ctx, const int* tokens, size_t n_tokens, bool preprocess_only);
OPENMINI_API int openmini_sample_token(openmini_context_t* ctx, float temperature, float top_p, int top_k);
/* logits of the last decoded token; the array stays valid until the next call on ctx */
OPENMINI_API openmini_error_t openmini_get_logits(openmini_context_t* ctx, float** logits, size_t* n_logits);
OPENMINI_API void openmini_free_result(openmini_result_t* result);
OPENMINI_API openmini_error_t openmini_get_stats(const openmini_context_t* ctx, openmini_stats_t* stats);
OPENMINI_API void openmini_reset_stats(openmini_context_t* ctx);
OPENMINI_API openmini_error_t openmini_set_log_callback(openmini_log_callback_t callback, void* user_data);

/* ---------------------------------------------------------------------------
 * Allocation-free paged attention (exported by the CUDA kernel library
 * openmini_v1_b200/_C*.so, not by the runtime library above). It has no
 * counterpart in the reference.
 *
 * For callers that cannot allocate device memory: code running inside a
 * custom allocator or memory-pool hook, plugins hosted by a runtime that owns
 * all device memory, and real-time paths where a cudaMalloc could block. The
 * caller passes only inputs and outputs; the split-KV partials live in one
 * fixed device array of OM_NOALLOC_SCRATCH_FLOATS fp32 values (16 MiB) that
 * every GPU loading the library holds until the process exits.
 *
 *   q            bf16 [rows, Hq, head_dim], row stride q_ld elements
 *   k/v_cache    bf16 [num_blocks, Hkv, 16, head_dim] (16-token pages)
 *   block_tables int32 [num_seqs, max_blocks]
 *   row_seq      int32 [rows] sequence of each query row
 *   row_ctx      int32 [rows] visible keys of each row (<= max_ctx)
 *   out          bf16 [rows, Hq, head_dim], row stride out_ld elements
 *   status       optional device int32; a bad block id, sequence index or a
 *                context past max_ctx / the block table sets it to 5
 *                (the access is skipped or clamped)
 * head_dim is 64 or 128; Hq / Hkv is 1, 2, 4, 5, 8 or 16.
 * A call needs rows * Hq * ceil(max_ctx / 512) * (head_dim + 2) floats of the
 * array; larger requests return OM_NOALLOC_TOO_LARGE. The first call on a
 * device looks up the array's address with that device current; make it
 * before any stream capture. Every call shares the array, so calls that
 * overlap on the GPU (other streams, other host threads) race: serialise them.
 * No cudaMalloc, cudaFree or allocating library routine is called.
 * ------------------------------------------------------------------------- */
#define OM_NOALLOC_SCRATCH_FLOATS (4u << 20)
enum {
  OM_NOALLOC_OK = 0,
  OM_NOALLOC_TOO_LARGE = 1,   /* request exceeds the fixed scratch array */
  OM_NOALLOC_BAD_ARGS = 2,    /* unsupported head_dim / GQA group / null pointer / bad size */
  OM_NOALLOC_CUDA_ERROR = 3,  /* symbol lookup or kernel launch failed */
};
struct CUstream_st;
OPENMINI_API int om_paged_attention_noalloc(const void* q, int q_ld, const void* k_cache, const void* v_cache,
                                            int num_blocks, int Hkv, int head_dim, const int* block_tables,
                                            int num_seqs, int max_blocks, const int* row_seq, const int* row_ctx,
                                            int rows, void* out, int out_ld, int Hq, int max_ctx, float scale,
                                            int* status, struct CUstream_st* stream);

#ifdef __cplusplus
}
#endif
