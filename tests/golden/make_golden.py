"""Generate the golden attention fixtures from the reference's own PyTorch modules.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/fast-gpu-asr

The reference package's ``__init__`` imports CuPy and TensorRT, so the script installs
a bare stub package whose ``__path__`` points at ``<reference>/src/fast_gpu_asr`` and
imports only the two attention modules, which need nothing but torch:

* ``src/fast_gpu_asr/export/model/zipformer/attention.py``
  (``RelPositionMultiheadAttentionWeights``, ``SelfAttention``, ``NonlinAttention``)
* ``src/fast_gpu_asr/export/model/parakeet/attention.py``
  (``RelPositionMultiHeadAttention``, ``RelPositionalEncoding``)

and, for ``positional_tables.npz``, the two positional encodings
(``RelPositionalEncoding``, ``CompactRelPositionalEncoding``, zipformer/attention.py:292-374).

The convolution fixtures (``conv_*.npz``) come from the two convolution modules,
``ConformerConvolution`` (``export/model/parakeet/parakeet.py:495-582``) and
``ConvolutionModule`` (``export/model/zipformer/zipformer.py:511-573``). Each module runs
twice on the same input: once with ONNX export simulated (``torch.onnx.is_in_onnx_export``
patched to True and ``torch.onnx.ops.symbolic`` replaced by a recorder), which captures
exactly the tensors the module hands to its TensorRT plugin - for Parakeet the depthwise
weights and bias with the BatchNorm folded in by the module's own export code - and once
eagerly, with the output projection set to the identity, which gives the plugin-boundary
output in fp32.

Each fixture stores the plugin-boundary inputs (the projections the modules feed to
their TensorRT plugins) and the module's eager output at that boundary. Output
projections are set to (an embedding of) the identity so the module output equals
the plugin output. All arrays are stored as float32 (fp16/bf16 values are exact in
float32). The GPU box never runs this script; it only reads the ``.npz`` files.
"""

from __future__ import annotations

import argparse
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def import_reference(reference: Path):
    pkg = types.ModuleType("fast_gpu_asr")
    pkg.__path__ = [str(reference / "src" / "fast_gpu_asr")]
    sys.modules["fast_gpu_asr"] = pkg
    from fast_gpu_asr.export.model.parakeet import attention as parakeet
    from fast_gpu_asr.export.model.zipformer import attention as zipformer

    return zipformer, parakeet


def import_reference_models():
    """The model modules holding the convolution modules (after import_reference)."""
    from fast_gpu_asr.export.model.parakeet import parakeet as parakeet_model
    from fast_gpu_asr.export.model.zipformer import zipformer as zipformer_model

    return zipformer_model, parakeet_model


def capture_plugin_inputs(module, x, lengths):
    """Run ``module`` as under ONNX export and return the tensors it passes to its plugin."""
    captured = {}

    def symbolic(name, inputs, attrs=None, **kwargs):
        captured["name"] = name
        captured["inputs"] = [t.detach().clone() for t in inputs]
        return torch.zeros(kwargs["shape"], dtype=kwargs["dtype"])

    saved = (torch.onnx.is_in_onnx_export, torch.onnx.ops.symbolic)
    torch.onnx.is_in_onnx_export = lambda: True
    torch.onnx.ops.symbolic = symbolic
    try:
        with torch.no_grad():
            module(x, lengths)
    finally:
        torch.onnx.is_in_onnx_export, torch.onnx.ops.symbolic = saved
    return captured


def conv_case(model_mod, kind, name, n, t, channels, kernel, seed, lengths) -> None:
    """Plugin-boundary inputs and eager fp32 output of one convolution module."""
    torch.manual_seed(seed)
    if kind == "parakeet":
        module = model_mod.ConformerConvolution(channels, kernel, True)
        out_proj = module.pointwise_conv2
        with torch.no_grad():
            bn = module.batch_norm
            bn.weight.uniform_(0.5, 1.5)
            bn.bias.normal_(0.0, 0.1)
            bn.running_mean.normal_(0.0, 0.2)
            bn.running_var.uniform_(0.5, 2.0)
    else:
        module = model_mod.ConvolutionModule(channels, kernel)
        out_proj = module.out_proj
    module.eval()
    embed_identity(out_proj)
    x = torch.randn(n, t, channels)
    lens = torch.tensor(lengths, dtype=torch.int32)
    captured = capture_plugin_inputs(module, x, lens)
    with torch.no_grad():
        eager = module(x, lens)
    px, plens, weight, bias = captured["inputs"]
    np.savez_compressed(
        HERE / f"{name}.npz", plugin=np.array(captured["name"]), x=f32(px),
        valid_lengths=plens.numpy().astype(np.int32), weight=f32(weight), bias=f32(bias),
        output=f32(eager))
    print(name, captured["name"], tuple(px.shape), tuple(weight.shape))


def suffix_mask(lengths, t):
    return (np.arange(t)[None, :] >= np.asarray(lengths)[:, None])


def embed_identity(linear: torch.nn.Linear) -> None:
    """out_proj weight [out, in] = identity on the first `in` outputs, zero bias."""
    with torch.no_grad():
        linear.weight.zero_()
        n = min(linear.weight.shape)
        linear.weight[:n, :n] = torch.eye(n)
        if linear.bias is not None:
            linear.bias.zero_()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float32)


def zipformer_case(zip_mod, name, dtype, n, t, embed, heads, qd, vd, pos_dim, seed,
                   lengths=None, xavier=False):
    """Weights module + two SelfAttention value applications + NonlinAttention."""
    dt = DTYPES[dtype]
    torch.manual_seed(seed)
    rng = np.random.default_rng(seed)
    weights_mod = zip_mod.RelPositionMultiheadAttentionWeights(embed, pos_dim, heads, qd, 4)
    self_a = zip_mod.SelfAttention(embed, heads, vd)
    self_b = zip_mod.SelfAttention(embed, heads, vd)
    att_dim = 3 * embed // 4
    nonlin = zip_mod.NonlinAttention(embed, att_dim)
    mods = (weights_mod, self_a, self_b, nonlin)
    with torch.no_grad():
        for m in mods:
            for lin in m.modules():
                if isinstance(lin, torch.nn.Linear):
                    if xavier:
                        torch.nn.init.xavier_uniform_(lin.weight)
                    else:
                        lin.weight.normal_(0.0, 0.25 / np.sqrt(lin.weight.shape[1]))
                    if lin.bias is not None:
                        lin.bias.zero_()
        embed_identity(self_a.out_proj)
        embed_identity(self_b.out_proj)
        embed_identity(nonlin.out_proj)
        # Make the gate y == 1 so NonlinAttention's output is the plugin output.
        nonlin.in_proj.weight[2 * att_dim :].zero_()
        nonlin.in_proj.bias[2 * att_dim :].fill_(1.0)
    for m in mods:
        m.to(dt)
    x = torch.from_numpy(rng.normal(0.0, 1.0, (n, t, embed)).astype(np.float32)).to(dt)
    pos_emb = torch.from_numpy(rng.normal(0.0, 1.0, (1, 2 * t - 1, pos_dim)).astype(np.float32)).to(dt)
    if lengths is None:
        lengths = rng.integers(max(1, t // 2), t + 1, size=n)
    mask = torch.from_numpy(suffix_mask(lengths, t))
    with torch.no_grad():
        projection = weights_mod.in_proj(x)
        position = weights_mod.linear_pos(pos_emb).reshape(1, 2 * t - 1, heads, 4)
        attn = weights_mod(x, pos_emb, mask)
        value_a = self_a.in_proj(x)
        value_b = self_b.in_proj(x)
        out_a = self_a(x, attn)[:, :, : heads * vd]
        out_b = self_b(x, attn)[:, :, : heads * vd]
        s, xv, _y = nonlin.in_proj(x).chunk(3, dim=2)
        nonlin_value = xv * torch.tanh(s)
        nonlin_out = nonlin(x, attn)[:, :, :att_dim]
    np.savez_compressed(
        HERE / f"{name}.npz",
        kind="zipformer", dtype=dtype, num_heads=heads, query_head_dim=qd,
        projection=f32(projection), position=f32(position), mask=mask.numpy(),
        lengths=np.asarray(lengths, np.int32), weights=f32(attn),
        value_a=f32(value_a), out_a=f32(out_a), value_b=f32(value_b), out_b=f32(out_b),
        nonlin_value=f32(nonlin_value), nonlin_out=f32(nonlin_out),
    )
    print("wrote", name, tuple(attn.shape))


def parakeet_case(par_mod, name, dtype, n, t, heads, head_dim, seed, lengths, use_bias=True):
    dt = DTYPES[dtype]
    torch.manual_seed(seed)
    rng = np.random.default_rng(seed)
    feat = heads * head_dim
    mod = par_mod.RelPositionMultiHeadAttention(heads, feat, use_bias)
    with torch.no_grad():
        torch.nn.init.xavier_uniform_(mod.linear_qkv.weight)
        torch.nn.init.xavier_uniform_(mod.linear_pos.weight)
        if use_bias:
            mod.linear_qkv.bias.normal_(0.0, 0.02)
        mod.pos_bias_u.normal_(0.0, 0.02 * 10)
        mod.pos_bias_v.normal_(0.0, 0.02 * 10)
        embed_identity(mod.linear_out)
    mod.to(dt)
    enc = par_mod.RelPositionalEncoding(feat, t)
    x = torch.from_numpy(rng.normal(0.0, 1.0, (n, t, feat)).astype(np.float32)).to(dt)
    pos_emb = enc(x)
    lens = torch.tensor(lengths, dtype=torch.int32)
    with torch.no_grad():
        qkv = mod.linear_qkv(x)
        position = mod.linear_pos(pos_emb.to(dt))
        out = mod(x, pos_emb, lens)
    np.savez_compressed(
        HERE / f"{name}.npz",
        kind="parakeet", dtype=dtype, num_heads=heads, head_dim=head_dim,
        scale=np.float32(1.0 / head_dim**0.5),
        qkv=f32(qkv), position=f32(position), content_bias=f32(mod.pos_bias_u),
        position_bias=f32(mod.pos_bias_v), valid_lengths=np.asarray(lengths, np.int32),
        output=f32(out),
    )
    print("wrote", name, tuple(out.shape))


def positional_tables(zip_mod, par_mod) -> None:
    """Row a7: the reference's positional tables, selected for sequence lengths shorter
    than and equal to the table's maximum (the forward pass slices the central 2T-1 rows)."""
    out = {}
    for model_dim, max_len, t in ((1024, 50, 50), (64, 400, 375)):
        enc = par_mod.RelPositionalEncoding(model_dim, max_len)
        out[f"parakeet_{model_dim}_{t}"] = f32(enc(torch.zeros(1, t, model_dim)))
    for embed_dim, max_len, t in ((48, 750, 750), (48, 800, 94)):
        enc = zip_mod.CompactRelPositionalEncoding(embed_dim, max_len)
        out[f"zipformer_{embed_dim}_{t}"] = f32(enc(torch.zeros(1, t, embed_dim)))
    np.savez_compressed(HERE / "positional_tables.npz", **out)
    print("wrote positional_tables", {k: v.shape for k, v in out.items()})


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", type=Path, required=True)
    args = parser.parse_args()
    zip_mod, par_mod = import_reference(args.reference)
    # fp32, N=2, T=100, E=192, 4 heads, qd 32, pd 4, vd 12, pos_dim 48,
    # Xavier-uniform projections from seed 0, N(0,1) inputs, lengths U[50,100].
    zipformer_case(zip_mod, "zipformer_config1_fp32", "float32", 2, 100, 192, 4, 32, 12, 48,
                   seed=0, xavier=True)
    zipformer_case(zip_mod, "zipformer_t65_fp16", "float16", 2, 65, 128, 4, 32, 12, 48,
                   seed=11, lengths=(65, 40))
    zipformer_case(zip_mod, "zipformer_t65_bf16", "bfloat16", 2, 65, 128, 4, 32, 12, 48,
                   seed=12, lengths=(51, 65))
    zipformer_case(zip_mod, "zipformer_h8_t40_bf16", "bfloat16", 2, 40, 256, 8, 32, 12, 48,
                   seed=13, lengths=(40, 9))
    parakeet_case(par_mod, "parakeet_h2_d64_t37_fp32", "float32", 2, 37, 2, 64, seed=21,
                  lengths=(37, 20))
    parakeet_case(par_mod, "parakeet_h2_d128_t50_fp16", "float16", 2, 50, 2, 128, seed=22,
                  lengths=(50, 31))
    parakeet_case(par_mod, "parakeet_h2_d128_t50_bf16", "bfloat16", 2, 50, 2, 128, seed=23,
                  lengths=(44, 0))
    parakeet_case(par_mod, "parakeet_h1_d128_t160_fp16", "float16", 1, 160, 1, 128, seed=24,
                  lengths=(137,))
    positional_tables(zip_mod, par_mod)
    zip_model, par_model = import_reference_models()
    conv_case(par_model, "parakeet", "conv_parakeet_k9_c64", 3, 41, 64, 9, seed=31,
              lengths=(41, 17, 0))
    conv_case(par_model, "parakeet", "conv_parakeet_k9_c38", 2, 23, 38, 9, seed=32,
              lengths=(23, 5))
    conv_case(zip_model, "zipformer", "conv_zipformer_k31_c48", 3, 70, 48, 31, seed=33,
              lengths=(70, 44, 1))
    conv_case(zip_model, "zipformer", "conv_zipformer_k15_c40", 2, 19, 40, 15, seed=34,
              lengths=(12, 19))


if __name__ == "__main__":
    main()
