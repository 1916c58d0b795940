"""Python face of the native decode engine (include/b200_engine.h).

Loads a QWENBIN1 model directory (config.json + model.w16a16.qbin or
model.w8a16.qbin), concatenates q/k/v and gate/up rows on the device, and
runs prefill + greedy decode (one persistent cooperative kernel for all
decode steps by default, or one CUDA graph replay per step).  Same model and weights as the
reference engine (reference src/qwen2.cpp); see csrc/engine.cu.
"""
from __future__ import annotations

import ctypes
import json
import os
import time

import numpy as np
import torch

from . import ABI, _check
from . import qbin

_p = ctypes.c_void_p
_i = ctypes.c_int


class EngineConfig(ctypes.Structure):
    _fields_ = [("hidden", _i), ("intermediate", _i), ("layers", _i), ("heads", _i),
                ("kv_heads", _i), ("vocab", _i), ("max_seq", _i), ("eps", ctypes.c_float),
                ("theta", ctypes.c_float), ("w8", _i)]


class EngineLayer(ctypes.Structure):
    _fields_ = [(n, _p) for n in ("qkv_w", "qkv_s", "qkv_b", "o_w", "o_s", "gate_up_w",
                                  "gate_up_s", "down_w", "down_s", "input_norm", "post_norm")]


for _name, (_args, _res) in {
    "b200_engine_create": ([ctypes.POINTER(_p), ctypes.POINTER(EngineConfig),
                            ctypes.POINTER(EngineLayer), _p, _p, _p], _i),
    "b200_engine_destroy": ([_p], _i),
    "b200_engine_prefill": ([_p, ctypes.POINTER(_i), _i], _i),
    "b200_engine_decode": ([_p, _i], _i),
    "b200_engine_tokens": ([_p, ctypes.POINTER(_i), _i], _i),
    "b200_engine_logits": ([_p, ctypes.POINTER(ctypes.c_uint16)], _i),
    "b200_engine_set_decode_mode": ([_p, _i], _i),
    "b200_engine_decode_mode": ([_p], _i),
    "b200_engine_device_status": ([_p, _i], _i),
    "b200_engine_set_trace": ([_p, _i], _i),
    "b200_engine_force_token": ([_p, _i], _i),
    "b200_engine_test_stall": ([_p, _i], _i),
    "b200_engine_read_trace": ([_p, _p], _i),
}.items():
    _fn = getattr(ABI, _name)
    _fn.argtypes = _args
    _fn.restype = _res


def _dev(a: np.ndarray, device):
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).to(device).view(torch.bfloat16)
    return torch.from_numpy(a.copy()).to(device)


DECODE_MODES = {"persistent": 0, "graph": 1}


class Engine:
    """Greedy batch-1 decoder on one GPU."""

    def __init__(self, model_dir: str, precision: str = "w8a16", max_seq: int = 256,
                 device="cuda", mode: str | None = None):
        cfg = json.load(open(os.path.join(model_dir, "config.json")))
        arch = qbin.load_archive(os.path.join(model_dir, qbin.ARCHIVE_NAMES[precision]))
        self.device = torch.device(device)
        self.w8 = precision == "w8a16"
        self.cfg = cfg
        keep = []  # device tensors referenced by the engine

        def t(name):
            x = _dev(arch[name], self.device)
            keep.append(x)
            return x

        def cat(names):
            x = torch.cat([_dev(arch[n], self.device) for n in names], 0).contiguous()
            keep.append(x)
            return x

        layers = (EngineLayer * cfg["num_hidden_layers"])()
        for i in range(cfg["num_hidden_layers"]):
            p = f"model.layers.{i}."
            a = p + "self_attn."
            m = p + "mlp."
            L = layers[i]
            L.qkv_w = cat([a + "q_proj.weight", a + "k_proj.weight", a + "v_proj.weight"]).data_ptr()
            L.qkv_b = cat([a + "q_proj.bias", a + "k_proj.bias", a + "v_proj.bias"]).data_ptr()
            L.o_w = t(a + "o_proj.weight").data_ptr()
            L.gate_up_w = cat([m + "gate_proj.weight", m + "up_proj.weight"]).data_ptr()
            L.down_w = t(m + "down_proj.weight").data_ptr()
            if self.w8:
                L.qkv_s = cat([a + f"{x}_proj.weight.scale" for x in "qkv"]).data_ptr()
                L.o_s = t(a + "o_proj.weight.scale").data_ptr()
                L.gate_up_s = cat([m + "gate_proj.weight.scale",
                                   m + "up_proj.weight.scale"]).data_ptr()
                L.down_s = t(m + "down_proj.weight.scale").data_ptr()
            L.input_norm = t(p + "input_layernorm.weight").data_ptr()
            L.post_norm = t(p + "post_attention_layernorm.weight").data_ptr()
        head = "lm_head.weight" if "lm_head.weight" in arch else "model.embed_tokens.weight"
        embed = t("model.embed_tokens.weight")
        if head != "model.embed_tokens.weight":
            raise ValueError("untied LM head is not supported by this engine")
        fnorm = t("model.norm.weight")
        self._keep = keep
        self.config = EngineConfig(cfg["hidden_size"], cfg["intermediate_size"],
                                   cfg["num_hidden_layers"], cfg["num_attention_heads"],
                                   cfg["num_key_value_heads"], cfg["vocab_size"], max_seq,
                                   cfg.get("rms_norm_eps", 1e-6), cfg.get("rope_theta", 1e6),
                                   1 if self.w8 else 0)
        self.stream = torch.cuda.Stream(device=self.device)
        self.handle = _p()
        _check(ABI.b200_engine_create(ctypes.byref(self.handle), ctypes.byref(self.config),
                                      layers, embed.data_ptr(), fnorm.data_ptr(),
                                      self.stream.cuda_stream), "engine_create")
        torch.cuda.synchronize()
        if mode is not None:
            self.set_mode(mode)

    @property
    def mode(self) -> str:
        m = ABI.b200_engine_decode_mode(self.handle)
        return {v: k for k, v in DECODE_MODES.items()}[m]

    def set_mode(self, mode: str) -> None:
        _check(ABI.b200_engine_set_decode_mode(self.handle, DECODE_MODES[mode]),
               "engine_set_decode_mode")

    def trace(self, barriers: int) -> None:
        """Records the persistent kernel's per-CTA phase timeline for the
        first `barriers` phases of the next decode calls."""
        _check(ABI.b200_engine_set_trace(self.handle, barriers), "engine_set_trace")
        self._trace_barriers = barriers

    def read_trace(self) -> np.ndarray:
        """[cta, phase, (staged, done, block landed, input arrived)] global-timer ns."""
        ctas = ABI.b200_engine_read_trace(self.handle, None)
        if ctas <= 0:
            return np.zeros((0, 0, 4), np.uint64)
        buf = np.zeros((ctas, self._trace_barriers, 4), np.uint64)
        rc = ABI.b200_engine_read_trace(self.handle, buf.ctypes.data)
        if rc < 0:
            _check(rc, "engine_read_trace")
        return buf

    def device_status(self, clear: bool = False) -> int:
        return ABI.b200_engine_device_status(self.handle, 1 if clear else 0)

    def generate(self, prompt, new_tokens: int):
        """(tokens, ttft_ms, decode_ms): prefill, then new_tokens-1 decode steps."""
        arr = (_i * len(prompt))(*prompt)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _check(ABI.b200_engine_prefill(self.handle, arr, len(prompt)), "engine_prefill")
        first = (_i * 1)()
        _check(ABI.b200_engine_tokens(self.handle, first, 1), "engine_tokens")
        t1 = time.perf_counter()
        _check(ABI.b200_engine_decode(self.handle, new_tokens - 1), "engine_decode")
        out = (_i * new_tokens)()
        _check(ABI.b200_engine_tokens(self.handle, out, new_tokens), "engine_tokens")
        t2 = time.perf_counter()
        return list(out), (t1 - t0) * 1e3, (t2 - t1) * 1e3

    def teacher_forced(self, prompt, tokens):
        """Follows `tokens` (another engine's greedy output for `prompt`):
        after the prefill and after each forced step, records this engine's
        argmax and the gap between its two largest BF16 logits.  Returns
        (argmax list, gap list), one entry per token of `tokens`."""
        arr = (_i * len(prompt))(*prompt)
        _check(ABI.b200_engine_prefill(self.handle, arr, len(prompt)), "engine_prefill")
        am, gaps = [], []

        def record():
            lg = self.logits().astype(np.uint32) << 16
            v = lg.view(np.float32)
            top = np.argpartition(-v, 1)[:2]
            a, b = sorted(v[top], reverse=True)
            am.append(int(np.flatnonzero(v == a)[0]))
            gaps.append(float(a - b))
        record()
        for t in tokens[:-1]:
            _check(ABI.b200_engine_force_token(self.handle, int(t)), "engine_force_token")
            _check(ABI.b200_engine_decode(self.handle, 1), "engine_decode")
            record()
        return am, gaps

    def logits(self) -> np.ndarray:
        buf = (ctypes.c_uint16 * self.config.vocab)()
        _check(ABI.b200_engine_logits(self.handle, buf), "engine_logits")
        return np.frombuffer(buf, dtype=np.uint16).copy()

    def close(self):
        if self.handle:
            ABI.b200_engine_destroy(self.handle)
            self.handle = _p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
