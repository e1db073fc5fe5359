"""Weight loading and high-level decode API for Qwen3-0.6B (B200 engine).

Drop-in counterpart of the upstream ``Model/Qwen06B_architecture.py``: the
same module constants, ``EXTENSION_ABI_VERSION``, ``load_weights``,
``_pack_layer_weights``, ``Decoder`` (``step`` / ``generate`` / ``reset`` /
``position``) and ``generate``, driving the ``qwen_megakernel_C`` extension
built from this package (``build.py``).  There is no CPU fallback: importing
this module without the built CUDA extension raises, as upstream does
(``Model/Qwen06B_architecture.py:31-94``).

Differences from upstream, all deliberate:
* misaligned weight or scratch pointers raise ``RuntimeError`` instead of
  being printed (the B200 kernel streams weights with 16-byte bulk copies);
* ``step`` raises if the device reports a failed launch (a -1 token), and
  ``generate`` likewise;
* ``load_weights("synthetic[:seed]")`` returns seeded random-init weights of
  the real architecture (``qwen_weights.synthetic_weights``); any other name
  goes to HF ``from_pretrained`` exactly as upstream;
* ``Decoder.generate_ids`` takes token ids and returns token ids, for callers
  without a tokenizer.
"""
from __future__ import annotations

import ctypes
import math
import os
import sys

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
if _HERE not in sys.path:
    sys.path.insert(0, _HERE)

try:
    import qwen_megakernel_C
except ImportError:
    qwen_megakernel_C = None

from qwen_weights import (HEAD_DIM, HIDDEN_SIZE, INTERMEDIATE_SIZE, KV_SIZE, MAX_SEQ_LEN,  # noqa: E402
                          NUM_KV_HEADS, NUM_LAYERS, Q_SIZE, ROPE_THETA, VOCAB_SIZE,
                          rope_tables, synthetic_weights)

EXTENSION_ABI_VERSION = 2

__all__ = ["EXTENSION_ABI_VERSION", "NUM_LAYERS", "NUM_KV_HEADS", "HEAD_DIM", "HIDDEN_SIZE",
           "INTERMEDIATE_SIZE", "Q_SIZE", "KV_SIZE", "MAX_SEQ_LEN", "VOCAB_SIZE", "ROPE_THETA",
           "load_weights", "Decoder", "generate"]


def _require_megakernel_op(op_name: str):
    """Return an op from the extension module (upstream :31-60)."""
    if qwen_megakernel_C is not None and hasattr(qwen_megakernel_C, op_name):
        return getattr(qwen_megakernel_C, op_name)
    namespace = getattr(torch.ops, "qwen_megakernel_C", None)
    if namespace is not None and hasattr(namespace, op_name):
        return getattr(namespace, op_name)
    raise RuntimeError(
        f"qwen_megakernel_C op '{op_name}' is unavailable: the B200 CUDA extension is not "
        f"built or not loadable for torch {torch.__version__}. Build it with "
        f"`python {os.path.join(_HERE, 'build.py')}`.")


def _assert_extension_compatibility() -> None:
    """Fail fast on a stale extension binary (upstream :63-91)."""
    if qwen_megakernel_C is None:
        return
    try:
        ext_abi = int(qwen_megakernel_C.abi_version())
    except Exception:
        ext_abi = None
    if ext_abi != EXTENSION_ABI_VERSION:
        built = getattr(qwen_megakernel_C, "built_torch_version", lambda: "unknown")()
        raise RuntimeError(
            f"Incompatible qwen_megakernel_C extension: expected ABI {EXTENSION_ABI_VERSION}, "
            f"got {ext_abi} (built against torch {built}); rebuild it.")


_assert_extension_compatibility()
_decode = _require_megakernel_op("decode")


_native = None


def _native_lib():
    """The C-ABI library (for the entry points the pybind module does not wrap)."""
    global _native
    if _native is None:
        path = os.path.join(_HERE, "libqwen_b200.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: build it with qwen0.6b_b200/build.py")
        L = ctypes.CDLL(path)
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.qwen_b200_decode_step_dev.restype = i
        L.qwen_b200_decode_step_dev.argtypes = [vp] * 22 + [i, i, i, ctypes.c_float, vp]
        L.qwen_b200_last_error.restype = i
        L.qwen_b200_last_error.argtypes = [ctypes.c_char_p, i]
        _native = L
    return _native


def load_weights(model_name: str = "Qwen/Qwen3-0.6B", verbose: bool = True):
    """Weights dict + tokenizer, in the upstream layout (upstream :97-174).

    ``model_name`` is a local checkpoint directory (or safetensors file), or a
    Hugging Face model id resolved through the local hub cache.  The tensors
    are read by the native safetensors reader and cast to fp16 on the device
    (``checkpoint.load_checkpoint``; upstream instantiates the transformers
    model for this); the tokenizer is the byte-level BPE of the checkpoint's
    ``tokenizer.json`` (``tokenizer.QwenTokenizer``), or None when the
    checkpoint has none.  ``"synthetic"`` or ``"synthetic:<seed>"`` gives
    seeded random-init weights and no tokenizer.
    """
    if model_name.startswith("synthetic"):
        seed = int(model_name.split(":", 1)[1]) if ":" in model_name else 0
        return synthetic_weights(seed=seed, device="cuda"), None

    from checkpoint import load_checkpoint, resolve_checkpoint
    from tokenizer import QwenTokenizer

    path = resolve_checkpoint(model_name)
    if verbose:
        print(f"Loading {model_name} from {path}...")
    weights = load_checkpoint(path, device="cuda")
    tok_dir = path if os.path.isdir(path) else os.path.dirname(path)
    tokenizer = (QwenTokenizer.from_dir(tok_dir)
                 if os.path.exists(os.path.join(tok_dir, "tokenizer.json")) else None)
    return weights, tokenizer


_FIELD_NAMES = ("input_layernorm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm", "o_proj",
                "post_attn_norm", "gate_proj", "up_proj", "down_proj")


def _pack_layer_weights(layer_weights: list) -> torch.Tensor:
    """int64 device tensor of 12 pointers per layer (11 weights + zero pad),
    16-byte aligned: the LDGLayerWeight table (upstream :177-202)."""
    n = len(_FIELD_NAMES)
    n_layers = len(layer_weights) // n
    if n_layers < 1 or len(layer_weights) != n_layers * n:
        raise ValueError(f"expected {n} weight tensors per layer, got {len(layer_weights)}")
    bad = []
    ptrs = []
    for li in range(n_layers):
        for j in range(n):
            t = layer_weights[li * n + j]
            if not (t.is_cuda and t.dtype == torch.float16 and t.is_contiguous()):
                raise ValueError(f"layer {li} {_FIELD_NAMES[j]}: need a contiguous CUDA fp16 tensor")
            if t.data_ptr() % 16:
                bad.append(f"layer {li} {_FIELD_NAMES[j]} ptr={t.data_ptr():#x}")
            ptrs.append(t.data_ptr())
        ptrs.append(0)
    if bad:
        raise RuntimeError("misaligned weight tensors (16-byte alignment required): " + "; ".join(bad))
    dev = layer_weights[0].device
    t = torch.zeros(len(ptrs) + 2, dtype=torch.int64, device=dev)
    off = ((16 - t.data_ptr() % 16) % 16) // 8
    t_al = t[off: off + len(ptrs)]
    t_al.copy_(torch.tensor(ptrs, dtype=torch.int64))
    assert t_al.data_ptr() % 16 == 0
    return t_al


class Decoder:
    """Stateful decoder over the B200 persistent decode kernel (upstream :205-382)."""

    def __init__(self, weights=None, tokenizer=None, model_name="Qwen/Qwen3-0.6B",
                 verbose: bool = True, num_layers: int | None = None):
        if weights is None:
            weights, tokenizer = load_weights(model_name, verbose=verbose)
        self.tokenizer = tokenizer
        self._position = 0
        self._weights = weights  # keep alive: the packed table holds raw pointers
        self._embed_weight = weights["embed_weight"]
        self._final_norm_weight = weights["final_norm_weight"]
        self._lm_head_weight = weights["lm_head_weight"]
        self._cos_table = weights["cos_table"]
        self._sin_table = weights["sin_table"]
        lw = weights["layer_weights"]
        self._num_layers = num_layers or len(lw) // 11
        self._layer_weights_packed = _pack_layer_weights(lw[: self._num_layers * 11])
        self._attn_scale = 1.0 / math.sqrt(HEAD_DIM)
        dev = self._embed_weight.device
        self._k_cache = torch.zeros(self._num_layers, NUM_KV_HEADS, MAX_SEQ_LEN, HEAD_DIM,
                                    dtype=torch.float16, device=dev)
        self._v_cache = torch.zeros_like(self._k_cache)
        f16 = dict(dtype=torch.float16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = dict(dtype=torch.int32, device=dev)
        self._hidden = torch.empty(HIDDEN_SIZE, **f16)
        self._act = torch.empty(Q_SIZE, **f32)
        self._res = torch.empty(HIDDEN_SIZE, **f32)
        self._q = torch.empty(Q_SIZE, **f16)
        self._k = torch.empty(KV_SIZE, **f16)
        self._v = torch.empty(KV_SIZE, **f16)
        self._attn_out = torch.empty(Q_SIZE, **f16)
        self._mlp_inter = torch.empty(INTERMEDIATE_SIZE, **f32)
        self._norm_out = torch.empty(HIDDEN_SIZE, **f32)
        self._fmax_vals = torch.empty(4096, **f32)
        self._fmax_idxs = torch.empty(4096, **i32)
        self._out_token = torch.empty(1, **i32)

    def _args(self):
        return (self._embed_weight, self._layer_weights_packed, self._final_norm_weight,
                self._lm_head_weight, self._cos_table, self._sin_table, self._k_cache,
                self._v_cache, self._hidden, self._act, self._res, self._q, self._k, self._v,
                self._attn_out, self._mlp_inter, self._norm_out, self._fmax_vals,
                self._fmax_idxs)

    def _raise_device_failure(self, what: str) -> None:
        status = int(qwen_megakernel_C.device_status(self._embed_weight.device.index or 0))
        raise RuntimeError(f"{what}: device-side failure, status word {status:#x}")

    def step(self, input_token_id: int | torch.Tensor) -> int:
        """Decode one token at the current position; returns the greedy next token."""
        result = _decode(int(input_token_id), *self._args(), self._num_layers, self._position,
                         MAX_SEQ_LEN, self._attn_scale)
        self._out_token.copy_(result)
        tok = int(result.item())
        if tok < 0:
            self._raise_device_failure("Decoder.step")
        self._position += 1
        return tok

    def reset(self):
        self._position = 0
        self._k_cache.zero_()
        self._v_cache.zero_()

    @property
    def position(self) -> int:
        return self._position

    def prefill(self, token_ids: list[int], max_rows: int = 256) -> None:
        """Parallel prefill (no upstream counterpart; upstream calls step() once
        per prompt token, :346-347): writes the K/V of token_ids at positions
        position .. position+len-1 with the batched tensor-core path, in steps
        of up to max_rows tokens, and advances the position past them.  The
        next step() / generate_nosync() continues from there."""
        if not token_ids:
            return
        if self._position + len(token_ids) > MAX_SEQ_LEN:
            raise ValueError("prefill would run past the KV cache")
        if getattr(self, "_prefiller", None) is None or self._prefiller.max_rows != max_rows:
            from batched import BatchedDecoder
            self._prefiller = BatchedDecoder(
                self._weights, num_seqs=1, max_rows=max_rows, num_layers=self._num_layers,
                device=self._embed_weight.device, k_pool=self._k_cache.unsqueeze(0),
                v_pool=self._v_cache.unsqueeze(0))
        # prefill_parallel feeds all but the last token of a prompt: append one.
        self._prefiller.prefill_parallel([list(token_ids) + [0]], starts=[self._position])
        self._position += len(token_ids)

    def generate_ids(self, ids: list[int], max_tokens: int = 100, reset: bool = True) -> list[int]:
        """Prefill ids[:-1] with step(), then generate_nosync from ids[-1]."""
        if reset:
            self.reset()
        for tid in ids[:-1]:
            self.step(tid)
        out = self.generate_nosync(ids[-1], max_tokens).cpu().tolist()
        if any(t < 0 for t in out):
            self._raise_device_failure("Decoder.generate_ids")
        return out

    def generate_nosync(self, first_token: int, num_steps: int) -> torch.Tensor:
        """Device-resident greedy loop from the current position; int32[num_steps] on device."""
        gen = _require_megakernel_op("generate_nosync")
        out = gen(int(first_token), int(num_steps), *self._args(), self._num_layers,
                  self._position, MAX_SEQ_LEN, self._attn_scale)
        self._position += num_steps
        return out

    def sample_nosync(self, first_token: int, num_steps: int, temperature: float = 1.0,
                      top_k: int = 0, top_p: float = 1.0, seed: int = 0) -> torch.Tensor:
        """Sampled counterpart of ``generate_nosync`` (no upstream counterpart;
        upstream is greedy only): from the current position, per token one
        decode step that reads its input token from device memory and writes
        the logits, and one sampling launch that writes the next input token
        (``sampling.py``: temperature, top-k, top-p as the transformers
        warpers filter, Gumbel-max draw keyed by (seed, position)).  Returns
        the device int32 tokens; no host synchronisation."""
        from sampling import SamplingParams, sample
        if self._position + num_steps > MAX_SEQ_LEN:
            raise ValueError(f"{num_steps} tokens from position {self._position} exceed {MAX_SEQ_LEN}")
        dev = self._embed_weight.device
        log = torch.empty(num_steps + 1, dtype=torch.int32, device=dev)
        log[0] = int(first_token)
        if getattr(self, "_logits", None) is None:
            self._logits = torch.empty(VOCAB_SIZE, dtype=torch.float32, device=dev)
        params = SamplingParams(temperature, top_k, top_p, seed)
        stream = torch.cuda.current_stream(dev).cuda_stream
        L = _native_lib()
        ptrs = [t.data_ptr() for t in self._args()]
        for n in range(num_steps):
            rc = L.qwen_b200_decode_step_dev(
                log[n:].data_ptr(), self._out_token.data_ptr(), self._logits.data_ptr(), *ptrs,
                self._num_layers, self._position, MAX_SEQ_LEN, self._attn_scale, ctypes.c_void_p(stream))
            if rc:
                buf = ctypes.create_string_buffer(512)
                L.qwen_b200_last_error(buf, 512)
                raise RuntimeError(f"qwen_b200_decode_step_dev: {buf.value.decode()}")
            sample(self._logits, params, offset=self._position, out=log[n + 1:n + 2])
            self._position += 1
        return log[1:]

    def sample_ids(self, ids: list[int], max_tokens: int = 100, temperature: float = 1.0,
                   top_k: int = 0, top_p: float = 1.0, seed: int = 0, reset: bool = True) -> list[int]:
        """Prefill ids[:-1] with step(), then ``sample_nosync`` from ids[-1]."""
        if reset:
            self.reset()
        for tid in ids[:-1]:
            self.step(tid)
        out = self.sample_nosync(ids[-1], max_tokens, temperature, top_k, top_p, seed).cpu().tolist()
        if any(t < 0 for t in out) or int(self._out_token.item()) < 0:
            self._raise_device_failure("Decoder.sample_ids")
        return out

    def generate(self, prompt: str, max_tokens: int = 100, temperature: float = 0.0,
                 top_k: int = 0, top_p: float = 1.0, seed: int = 0) -> str:
        """Greedy as upstream (temperature 0, the default), else sampled."""
        self.reset()
        ids = self.tokenizer.encode(prompt, add_special_tokens=True)
        if temperature > 0.0 and top_k != 1:
            out = self.sample_ids(ids, max_tokens, temperature, top_k, top_p, seed, reset=False)
        else:
            out = self.generate_ids(ids, max_tokens, reset=False)
        eos = self.tokenizer.eos_token_id
        if eos in out:
            out = out[: out.index(eos)]
        return self.tokenizer.decode(out, skip_special_tokens=True)


def generate(prompt: str, max_tokens: int = 50, verbose: bool = True) -> str:
    """One-shot convenience: load model, generate, return text (upstream :385-387)."""
    return Decoder(verbose=verbose).generate(prompt, max_tokens)
