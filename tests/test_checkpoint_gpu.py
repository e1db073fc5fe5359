"""Checkpoint loading on the GPU (qwen0.6b_b200/checkpoint.py over the native
reader of include/qwen_b200_loader.h).

* BF16 / F32 / F16 tensors land as fp16 bit-identical to torch's
  ``.to(torch.float16)`` (round to nearest even, overflow to inf, subnormals),
  across the 16 MiB staging chunks and ragged tails.
* A 2-layer Qwen3 checkpoint written by transformers (bf16, tied embedding)
  loads bit-identically to upstream's own route,
  ``AutoModelForCausalLM.from_pretrained(path, float16).state_dict()``
  (Model/Qwen06B_architecture.py:122-127), and ``Decoder(model_name=path)``
  decodes the same tokens as a Decoder over those upstream tensors.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

st = pytest.importorskip("safetensors.torch")


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int16).cpu()


def test_device_cast_matches_torch(tmp_path):
    from checkpoint import SafetensorsFile
    g = torch.Generator().manual_seed(0)
    edge = torch.tensor([0.0, -0.0, 1.0, -2.5, 65504.0, 65519.0, 65520.0, -65520.0, 1e5, float("inf"),
                         -float("inf"), 6.1e-5, 6.09e-5, 5.96e-8, 2.98e-8, 2.99e-8, 1e-10, -1e-10, 3.14159])
    big = torch.randn(9_000_011, generator=g) * torch.exp(4 * torch.randn(9_000_011, generator=g))
    xs = torch.cat([edge, big])
    tensors = {"bf16": xs.bfloat16(), "f32": xs[:4_500_007].clone(), "f16": xs[:1001].half(),
               "nan": torch.tensor([float("nan"), 1.0]).bfloat16()}
    p = str(tmp_path / "cast.safetensors")
    st.save_file(tensors, p)
    with SafetensorsFile(p) as f:
        for name, t in tensors.items():
            out = torch.empty(t.numel(), dtype=torch.float16, device="cuda")
            f.load_f16(name, out)
            torch.cuda.synchronize()
            want = t.to(torch.float16).view(-1)
            if name == "nan":
                assert bool(torch.isnan(out[0])) and float(out[1]) == 1.0
                continue
            assert torch.equal(_bits(out), _bits(want)), name


def test_load_rejects_bad_destination(tmp_path):
    from checkpoint import SafetensorsFile
    p = str(tmp_path / "x.safetensors")
    st.save_file({"x": torch.zeros(8), "i": torch.zeros(2, dtype=torch.int32)}, p)
    with SafetensorsFile(p) as f:
        with pytest.raises(ValueError):
            f.load_f16("x", torch.empty(7, dtype=torch.float16, device="cuda"))
        with pytest.raises(RuntimeError, match="not F16, BF16 or F32"):
            f.load_f16("i", torch.empty(2, dtype=torch.float16, device="cuda"))


@pytest.fixture(scope="module")
def hf_checkpoint(tmp_path_factory):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Qwen3Config(
        vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=2,
        num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1e6, rms_norm_eps=1e-6,
        max_position_embeddings=2048, tie_word_embeddings=True)
    torch.manual_seed(0)
    model = transformers.Qwen3ForCausalLM(cfg)
    with torch.no_grad():
        for n, p in model.named_parameters():
            if "norm" in n:
                p.normal_(1.0, 0.1)  # non-trivial norm weights, so a mix-up shows
    d = tmp_path_factory.mktemp("qwen3_2l")
    model.to(torch.bfloat16).save_pretrained(str(d))
    del model
    try:
        ref = transformers.AutoModelForCausalLM.from_pretrained(str(d), dtype=torch.float16)
    except TypeError:
        ref = transformers.AutoModelForCausalLM.from_pretrained(str(d), torch_dtype=torch.float16)
    sd = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    return str(d), sd


def test_checkpoint_equals_upstream_transformers_route(hf_checkpoint):
    from checkpoint import HF_LAYER_NAMES, load_checkpoint
    path, sd = hf_checkpoint
    w = load_checkpoint(path)
    assert w["lm_head_weight"].data_ptr() == w["embed_weight"].data_ptr()  # tied, as upstream
    assert torch.equal(_bits(w["embed_weight"]), _bits(sd["model.embed_tokens.weight"]))
    assert torch.equal(_bits(w["final_norm_weight"]), _bits(sd["model.norm.weight"]))
    assert len(w["layer_weights"]) == 22
    for li in range(2):
        for j, n in enumerate(HF_LAYER_NAMES):
            got = w["layer_weights"][li * 11 + j]
            assert got.is_contiguous() and got.data_ptr() % 256 == 0
            assert torch.equal(_bits(got), _bits(sd[f"model.layers.{li}.{n}"])), (li, n)


def test_decoder_from_checkpoint_path(hf_checkpoint):
    from checkpoint import HF_LAYER_NAMES
    from Qwen06B_architecture import Decoder
    from qwen_weights import rope_tables
    path, sd = hf_checkpoint
    a = Decoder(model_name=path, verbose=False)
    assert a.tokenizer is None and a._num_layers == 2
    cos, sin = rope_tables()
    wref = dict(embed_weight=sd["model.embed_tokens.weight"].cuda(),
                layer_weights=[sd[f"model.layers.{li}.{n}"].cuda().contiguous()
                               for li in range(2) for n in HF_LAYER_NAMES],
                final_norm_weight=sd["model.norm.weight"].cuda(), cos_table=cos.cuda(), sin_table=sin.cuda())
    wref["lm_head_weight"] = wref["embed_weight"]
    b = Decoder(weights=wref, verbose=False)
    prompt = [11, 2000, 151000, 7, 99]
    assert a.generate_ids(prompt, 6) == b.generate_ids(prompt, 6)
