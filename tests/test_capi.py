"""The C ABI (include/openmini_b200.h) called through ctypes from the runtime
library: load a preset model, generate, drive decode / logits / sample by hand,
stats, log callback, error codes."""
import ctypes as C

import torch

from openmini_v1_b200 import _native


class Config(C.Structure):
    _fields_ = [("n_ctx", C.c_uint32), ("n_batch", C.c_uint32), ("n_threads", C.c_uint32),
                ("gpu_device_id", C.c_int), ("quant_type", C.c_char * 16), ("enable_kv_cache", C.c_bool),
                ("enable_flash_attn", C.c_bool), ("kv_cache_size_mb", C.c_uint32), ("use_bitnet_lut", C.c_bool),
                ("lut_block_size", C.c_uint32), ("rope_scaling", C.c_float), ("rope_freq_base", C.c_float),
                ("rope_freq_scale", C.c_float)]


class Result(C.Structure):
    _fields_ = [("tokens", C.POINTER(C.c_int)), ("n_tokens", C.c_size_t), ("text", C.c_char_p),
                ("duration_us", C.c_uint64), ("prompt_tokens", C.c_uint64), ("output_tokens", C.c_uint64),
                ("tokens_per_second", C.c_float), ("prompt_processing_us", C.c_float),
                ("token_generation_us", C.c_float)]


class Info(C.Structure):
    _fields_ = [("n_params", C.c_size_t), ("n_layers", C.c_size_t), ("n_head", C.c_size_t),
                ("n_head_kv", C.c_size_t), ("n_embd", C.c_size_t), ("n_vocab", C.c_size_t), ("n_ff", C.c_size_t),
                ("type", C.c_char * 64), ("quantization", C.c_char * 16)]


class Stats(C.Structure):
    _fields_ = [("total_prompt_us", C.c_uint64), ("total_gen_us", C.c_uint64), ("total_tokens", C.c_uint64),
                ("tokens_per_second", C.c_float), ("memory_used_mb", C.c_float), ("gpu_memory_used_mb", C.c_float),
                ("cache_hit_rate", C.c_uint32), ("n_prompt_tokens_processed", C.c_size_t),
                ("n_tokens_generated", C.c_size_t)]


def test_c_abi_end_to_end():
    lib = C.CDLL(_native.rt().__file__)
    lib.openmini_version.restype = C.c_char_p
    assert lib.openmini_init() == 0
    assert lib.openmini_version().decode().startswith("0.")
    logs = []
    CB = C.CFUNCTYPE(None, C.c_int, C.c_char_p, C.c_void_p)
    cb = CB(lambda lvl, txt, u: logs.append((lvl, txt.decode())))
    assert lib.openmini_set_log_callback(cb, None) == 0
    cfg = Config(n_ctx=256, gpu_device_id=-1, quant_type=b"bf16")
    model = C.c_void_p()
    assert lib.openmini_load_model(b"preset:tiny", C.byref(cfg), C.byref(model)) == 0
    assert any("loaded" in t for _, t in logs)
    info = Info()
    assert lib.openmini_model_info(model, C.byref(info)) == 0
    assert info.n_layers == 2 and info.n_vocab == 32000 and info.n_embd == 256
    ctx = C.c_void_p()
    assert lib.openmini_new_context(model, C.byref(ctx)) == 0
    res = Result()
    assert lib.openmini_generate(ctx, b"hello", 6, C.c_float(0.0), C.c_float(1.0), 0, C.byref(res)) == 0
    gen = [res.tokens[i] for i in range(res.n_tokens)]
    assert res.n_tokens == 6 and res.prompt_tokens == len("hello") + 1
    lib.openmini_free_result(C.byref(res))
    # the same greedy continuation driven by hand: decode -> logits argmax -> sample -> decode
    assert lib.openmini_reset_context(ctx) == 0
    from openmini_v1_b200.engine.tokenizer import ByteTokenizer
    prompt = ByteTokenizer().encode("hello")
    arr = (C.c_int * len(prompt))(*prompt)
    assert lib.openmini_decode(ctx, arr, len(prompt), False) == 0
    lp, n = C.POINTER(C.c_float)(), C.c_size_t()
    assert lib.openmini_get_logits(ctx, C.byref(lp), C.byref(n)) == 0 and n.value == 32000
    first = int(torch.tensor([lp[i] for i in range(n.value)]).argmax())
    t = lib.openmini_sample_token(ctx, C.c_float(0.0), C.c_float(1.0), 0)
    assert t == first == gen[0]
    one = (C.c_int * 1)(t)
    assert lib.openmini_decode(ctx, one, 1, False) == 0
    assert lib.openmini_sample_token(ctx, C.c_float(0.0), C.c_float(1.0), 0) == gen[1]
    st = Stats()
    assert lib.openmini_get_stats(ctx, C.byref(st)) == 0 and st.n_tokens_generated == 6
    # errors: context overflow, bad model path
    big = (C.c_int * 400)(*([5] * 400))
    assert lib.openmini_decode(ctx, big, 400, True) == -9
    assert lib.openmini_load_model(b"/nonexistent.gguf", C.byref(cfg), C.byref(C.c_void_p())) == -3
    lib.openmini_free_context(ctx)
    lib.openmini_free_model(model)
    lib.openmini_set_log_callback(None, None)
