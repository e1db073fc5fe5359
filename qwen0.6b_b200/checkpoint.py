"""Qwen3-0.6B checkpoints (safetensors) into the upstream ``load_weights`` dict.

Replaces the Hugging Face model instantiation of upstream ``load_weights``
(``Model/Qwen06B_architecture.py:97-174``): upstream builds an
``AutoModelForCausalLM`` with ``torch_dtype=torch.float16`` on the GPU and
takes its ``state_dict()``; here the safetensors files are read by the native
reader of ``libqwen_b200.so`` (``include/qwen_b200_loader.h``), streamed into
one device arena and cast to fp16 on the device with the same
round-to-nearest-even cast torch applies.  No transformers import, no model
object, and no second copy of the weights on the device.

The returned dict has upstream's keys and layouts: ``embed_weight``,
``layer_weights`` (11 tensors per layer in ``LDGLayerWeight`` order, HF
``[out, in]`` row-major), ``final_norm_weight``, ``lm_head_weight`` (the
embedding itself when the checkpoint ties them, as Qwen3-0.6B does:
``:163-170``) and the fp16 RoPE tables (``:134-142``).
"""
from __future__ import annotations

import ctypes
import json
import os

import torch

from qwen_weights import (HEAD_DIM, HIDDEN_SIZE, INTERMEDIATE_SIZE, KV_SIZE, LAYER_FIELDS,
                          MAX_SEQ_LEN, NUM_KV_HEADS, NUM_LAYERS, NUM_Q_HEADS, Q_SIZE, RMS_EPS,
                          ROPE_THETA, VOCAB_SIZE, rope_tables)

_PKG = os.path.dirname(os.path.abspath(__file__))
_lib = None

# HF parameter names of one decoder layer, in LDGLayerWeight order.
HF_LAYER_NAMES = ("input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
                  "self_attn.v_proj.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
                  "self_attn.o_proj.weight", "post_attention_layernorm.weight",
                  "mlp.gate_proj.weight", "mlp.up_proj.weight", "mlp.down_proj.weight")

ST_F16, ST_BF16, ST_F32, ST_OTHER = range(4)
_DTYPE_NAMES = {ST_F16: "F16", ST_BF16: "BF16", ST_F32: "F32", ST_OTHER: "other"}

# The architecture the decode kernels are built for (config.json keys).
EXPECTED_CONFIG = {
    "hidden_size": HIDDEN_SIZE, "intermediate_size": INTERMEDIATE_SIZE,
    "num_attention_heads": NUM_Q_HEADS, "num_key_value_heads": NUM_KV_HEADS,
    "head_dim": HEAD_DIM, "vocab_size": VOCAB_SIZE,
}


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = os.path.join(_PKG, "libqwen_b200.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with qwen0.6b_b200/build.py")
        L = ctypes.CDLL(path)
        vp, i, ll, cp = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_char_p
        L.qwen_b200_st_open.restype = i
        L.qwen_b200_st_open.argtypes = [cp, ctypes.POINTER(vp)]
        L.qwen_b200_st_close.restype = None
        L.qwen_b200_st_close.argtypes = [vp]
        L.qwen_b200_st_num_tensors.restype = i
        L.qwen_b200_st_num_tensors.argtypes = [vp]
        L.qwen_b200_st_find.restype = i
        L.qwen_b200_st_find.argtypes = [vp, cp]
        L.qwen_b200_st_info.restype = i
        L.qwen_b200_st_info.argtypes = [vp, i, ctypes.POINTER(cp), ctypes.POINTER(i), ctypes.POINTER(i),
                                        ctypes.POINTER(ll), ctypes.POINTER(ll)]
        L.qwen_b200_st_metadata.restype = cp
        L.qwen_b200_st_metadata.argtypes = [vp, cp]
        L.qwen_b200_st_read_host.restype = i
        L.qwen_b200_st_read_host.argtypes = [vp, i, vp, ll]
        L.qwen_b200_st_load_f16.restype = i
        L.qwen_b200_st_load_f16.argtypes = [vp, i, vp, vp]
        L.qwen_b200_last_error.restype = i
        L.qwen_b200_last_error.argtypes = [ctypes.c_char_p, i]
        _lib = L
    return _lib


def _check(rc: int, what: str) -> None:
    if rc:
        buf = ctypes.create_string_buffer(1024)
        lib().qwen_b200_last_error(buf, 1024)
        raise RuntimeError(f"{what} failed (code {rc}): {buf.value.decode(errors='replace')}")


class SafetensorsFile:
    """One safetensors file, read by the native reader."""

    def __init__(self, path: str):
        self.path = path
        h = ctypes.c_void_p()
        _check(lib().qwen_b200_st_open(os.fsencode(path), ctypes.byref(h)), f"opening {path}")
        self._h = h
        self._info = {}
        for i in range(lib().qwen_b200_st_num_tensors(h)):
            name, dt, nd = ctypes.c_char_p(), ctypes.c_int(), ctypes.c_int()
            shape, nbytes = (ctypes.c_longlong * 8)(), ctypes.c_longlong()
            _check(lib().qwen_b200_st_info(h, i, ctypes.byref(name), ctypes.byref(dt), ctypes.byref(nd),
                                           shape, ctypes.byref(nbytes)), f"{path}: tensor {i}")
            self._info[name.value.decode()] = (i, dt.value, tuple(shape[:nd.value]), nbytes.value)

    def close(self) -> None:
        if self._h is not None:
            lib().qwen_b200_st_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def names(self) -> list[str]:
        return list(self._info)

    def __contains__(self, name: str) -> bool:
        return name in self._info

    def dtype(self, name: str) -> str:
        return _DTYPE_NAMES[self._info[name][1]]

    def shape(self, name: str) -> tuple:
        return self._info[name][2]

    def metadata(self, key: str) -> str | None:
        v = lib().qwen_b200_st_metadata(self._h, key.encode())
        return None if v is None else v.decode()

    def read_bytes(self, name: str) -> bytes:
        """The tensor's raw bytes as stored (host only, no CUDA)."""
        i, _, _, n = self._info[name]
        buf = ctypes.create_string_buffer(max(1, n))
        _check(lib().qwen_b200_st_read_host(self._h, i, buf, n), f"{self.path}: reading {name}")
        return buf.raw[:n]

    def load_f16(self, name: str, out: torch.Tensor, stream: torch.cuda.Stream | None = None) -> None:
        """Tensor `name` as fp16 into the contiguous CUDA fp16 tensor `out`
        (enqueued on `stream`, default the current stream)."""
        i, _, shape, _ = self._info[name]
        numel = 1
        for s in shape:
            numel *= s
        if not (out.is_cuda and out.dtype == torch.float16 and out.is_contiguous() and out.numel() == numel):
            raise ValueError(f"{name}: need a contiguous CUDA fp16 tensor of {numel} elements")
        st = stream if stream is not None else torch.cuda.current_stream(out.device)
        with torch.cuda.device(out.device):
            _check(lib().qwen_b200_st_load_f16(self._h, i, ctypes.c_void_p(out.data_ptr()),
                                               ctypes.c_void_p(st.cuda_stream)), f"{self.path}: loading {name}")


def checkpoint_files(path: str) -> list[str]:
    """The safetensors files of a checkpoint: `path` itself, or those named by
    ``model.safetensors.index.json`` in a directory, else every
    ``*.safetensors`` there."""
    if os.path.isfile(path):
        return [path]
    if not os.path.isdir(path):
        raise FileNotFoundError(f"no checkpoint at {path}")
    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, n) for n in files]
    files = sorted(n for n in os.listdir(path) if n.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"{path} holds no .safetensors file")
    return [os.path.join(path, n) for n in files]


def read_config(path: str) -> dict:
    """config.json beside the checkpoint ({} when absent), checked against the
    architecture the kernels implement."""
    d = path if os.path.isdir(path) else os.path.dirname(path)
    cfg_path = os.path.join(d, "config.json")
    if not os.path.exists(cfg_path):
        return {}
    with open(cfg_path) as f:
        cfg = json.load(f)
    bad = {k: (cfg[k], v) for k, v in EXPECTED_CONFIG.items() if k in cfg and cfg[k] != v}
    if "rms_norm_eps" in cfg and abs(float(cfg["rms_norm_eps"]) - RMS_EPS) > 1e-12:
        bad["rms_norm_eps"] = (cfg["rms_norm_eps"], RMS_EPS)
    if bad:
        raise ValueError(f"{cfg_path}: not the Qwen3-0.6B geometry these kernels implement "
                         f"(key: (checkpoint, expected)) {bad}")
    return cfg


def _rope_theta(cfg: dict) -> float:
    if "rope_theta" in cfg:
        return float(cfg["rope_theta"])
    rp = cfg.get("rope_parameters") or {}
    return float(rp.get("rope_theta", ROPE_THETA))


def load_checkpoint(path: str, device: str | torch.device = "cuda", num_layers: int | None = None,
                    max_seq_len: int = MAX_SEQ_LEN) -> dict:
    """Weights dict (upstream ``load_weights`` layout) from a safetensors
    checkpoint file or directory.  Every weight lives in one fp16 device
    allocation, each tensor starting on a 256-byte boundary."""
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("load_checkpoint loads onto a CUDA device")
    cfg = read_config(path)
    n_layers = num_layers or int(cfg.get("num_hidden_layers", NUM_LAYERS))
    files = [SafetensorsFile(p) for p in checkpoint_files(path)]
    try:
        where = {}
        for f in files:
            for n in f.names():
                where.setdefault(n, f)
        plan = [("model.embed_tokens.weight", (VOCAB_SIZE, HIDDEN_SIZE))]
        for li in range(n_layers):
            for hf, (_, shape) in zip(HF_LAYER_NAMES, LAYER_FIELDS):
                plan.append((f"model.layers.{li}.{hf}", shape))
        plan.append(("model.norm.weight", (HIDDEN_SIZE,)))
        tied = bool(cfg.get("tie_word_embeddings", "lm_head.weight" not in where))
        if not tied:
            plan.append(("lm_head.weight", (VOCAB_SIZE, HIDDEN_SIZE)))
        missing = [n for n, _ in plan if n not in where]
        if missing:
            raise KeyError(f"checkpoint {path} lacks {len(missing)} tensors, e.g. {missing[:3]}")
        for n, shape in plan:
            if where[n].shape(n) != shape:
                raise ValueError(f"{n}: shape {where[n].shape(n)}, expected {shape}")
            if where[n].dtype(n) == "other":
                raise ValueError(f"{n}: stored as an unsupported dtype (need F16, BF16 or F32)")
        offs, total = [], 0
        for _, shape in plan:
            numel = 1
            for s in shape:
                numel *= s
            offs.append((total, numel))
            total += (numel + 127) // 128 * 128
        arena = torch.empty(total, dtype=torch.float16, device=dev)
        views = {}
        stream = torch.cuda.current_stream(dev)
        for (n, shape), (o, numel) in zip(plan, offs):
            t = arena[o:o + numel].view(shape)
            where[n].load_f16(n, t, stream)
            views[n] = t
        stream.synchronize()
    finally:
        for f in files:
            f.close()
    embed = views["model.embed_tokens.weight"]
    layer_weights = [views[f"model.layers.{li}.{hf}"] for li in range(n_layers) for hf in HF_LAYER_NAMES]
    cos, sin = rope_tables(max_seq_len, theta=_rope_theta(cfg))
    return dict(embed_weight=embed, layer_weights=layer_weights, final_norm_weight=views["model.norm.weight"],
                lm_head_weight=embed if tied else views["lm_head.weight"],
                cos_table=cos.to(dev), sin_table=sin.to(dev), arena=arena)


def resolve_checkpoint(model_name: str) -> str:
    """A local checkpoint directory or file for `model_name`: the path itself
    when it exists, else the Hugging Face hub cache snapshot (downloaded when
    the hub is reachable)."""
    if os.path.exists(model_name):
        return model_name
    try:
        from huggingface_hub import snapshot_download
    except ImportError as e:
        raise FileNotFoundError(f"{model_name} is not a local path and huggingface_hub is missing") from e
    patterns = ["*.safetensors", "*.json", "merges.txt", "vocab.json"]
    try:
        return snapshot_download(model_name, allow_patterns=patterns, local_files_only=True)
    except Exception:
        return snapshot_download(model_name, allow_patterns=patterns)
