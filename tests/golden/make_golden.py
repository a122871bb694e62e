"""Generate the golden fixtures under tests/golden from the reference itself.

Run once in a container that has the lite-ssm reference checked out (its path is
given with --reference). Nothing at test time reads the reference: every fixture
written here is committed, and the tests only read these files.

What is pinned, and by which reference code:
  int4_pack.npz      tools/export_mamba2.py:68-103 `quantize_int4_block32` applied to
                     seeded fp16 blocks (incl. all-zero, tie-at-.5 and clamp-edge blocks).
  layout_130m_*.bin  tools/ssm_format.py:316-340 `plan_layout` (header + tensor index
                     bytes) for the mamba2-130m state_dict (219 tensors, embedding
                     payload at offset 17600: tests/test_mmap_loader.cpp:64-95),
                     fp16 and int4 variants, plus a JSON table of (name, dtype, shape,
                     offset, nbytes).
  tiny_*.ssm         tools/export_mamba2.py:162-229 `collect_tensors` + `write_ssm` on
                     small random-init HF Mamba2ForCausalLM models (fp16 and int4).
  tiny_*_hf.npz      HF transformers' Mamba2ForCausalLM (the ground truth used by the
                     reference's own parity test, tools/dump_parity.py:26-70) run in fp32
                     on exactly the weights stored in the .ssm file: last-prompt-token
                     logits, greedy token ids and per-step logits.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def load_reference_tools(ref: Path):
    sys.path.insert(0, str(ref / "tools"))
    import ssm_format as fmt  # noqa: E402
    import export_mamba2 as exp  # noqa: E402
    return fmt, exp


def make_int4_pack(exp) -> None:
    g = torch.Generator().manual_seed(1234)
    N, K = 24, 256
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.float16)
    w[0, 0:32] = 0.0                                    # all-zero block -> clamp_min path
    w[1, 0:32] = torch.linspace(-1, 1, 32).to(torch.float16)
    w[2, 32:64] = torch.tensor([7.0, 3.5, -3.5, 2.5, -2.5, 0.5, -0.5, 1.5] * 4).to(torch.float16)  # ties
    w[3, 64:96] = torch.tensor([-7.0] + [8.0 / 7.0 * 7.0] * 31).to(torch.float16)               # clamp edges
    blob = exp.quantize_int4_block32(w)
    packed = np.frombuffer(blob[: N * K // 2], dtype=np.uint8).reshape(N, K // 2)
    scales = np.frombuffer(blob[N * K // 2:], dtype=np.uint16).reshape(N, K // 32)
    np.savez_compressed(HERE / "int4_pack.npz", w_f16=w.numpy().view(np.uint16), packed=packed, scales=scales)


def hf_config(d_model, n_layer, d_state, head_dim, n_groups, vocab, chunk, expand=2):
    from transformers import Mamba2Config
    d_inner = expand * d_model
    return Mamba2Config(
        vocab_size=vocab, hidden_size=d_model, num_hidden_layers=n_layer, state_size=d_state,
        expand=expand, head_dim=head_dim, num_heads=d_inner // head_dim, n_groups=n_groups,
        conv_kernel=4, chunk_size=chunk, use_conv_bias=True, use_bias=False,
        tie_word_embeddings=True, layer_norm_epsilon=1e-5, residual_in_fp32=True,
    )


def make_layout_130m(fmt, exp) -> None:
    from transformers import Mamba2ForCausalLM
    cfg = hf_config(768, 24, 128, 64, 1, 50288, 256)
    with torch.device("meta"):
        model = Mamba2ForCausalLM(cfg)
    sd = model.state_dict()
    hp = exp.hparams_from_config(cfg)
    for quant in ("fp16", "int4"):
        entries = []
        for name, t in sd.items():
            shape = tuple(t.shape)
            if quant == "int4" and exp.is_int4_quantizable(name, shape):
                entries.append(fmt.TensorEntry(name=name, dtype=fmt.DTYPE_INT4_B32, shape=shape))
            else:
                entries.append(fmt.TensorEntry(name=name, dtype=fmt.DTYPE_F16, shape=shape))
        plan = fmt.plan_layout(hp, entries)
        (HERE / f"layout_130m_{quant}.bin").write_bytes(plan.header + plan.index_blob)
        table = [dict(name=e.name, dtype=e.dtype, shape=list(e.shape), offset=e.offset, nbytes=e.nbytes)
                 for e in entries]
        (HERE / f"layout_130m_{quant}.json").write_text(json.dumps(dict(
            data_offset=plan.data_offset, n_tensors=len(entries), tensors=table)))


def dequant_int4(blob: bytes, N: int, K: int) -> torch.Tensor:
    packed = np.frombuffer(blob[: N * K // 2], dtype=np.uint8).reshape(N, K // 2).astype(np.int32)
    scales = np.frombuffer(blob[N * K // 2:], dtype=np.float16).reshape(N, K // 32).astype(np.float32)
    lo = packed & 0xF
    hi = packed >> 4
    q = np.empty((N, K), dtype=np.int32)
    q[:, 0::2] = lo
    q[:, 1::2] = hi
    q = np.where(q < 8, q, q - 16).astype(np.float32)
    return torch.from_numpy(q * np.repeat(scales, 32, axis=1))


def make_tiny(fmt, exp, tag, cfg_kwargs, seed, prompt_len, n_new) -> None:
    from transformers import Mamba2ForCausalLM
    torch.manual_seed(seed)
    cfg = hf_config(**cfg_kwargs)
    model = Mamba2ForCausalLM(cfg).eval()
    # Make the random init better conditioned for a parity test: unit-scale
    # embeddings and 1/sqrt(fan_in) linears keep the residual stream in fp16 range.
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("in_proj.weight") or name.endswith("out_proj.weight"):
                p.copy_(torch.randn_like(p) / np.sqrt(p.shape[1]))
            elif name.endswith("embeddings.weight"):
                p.copy_(torch.randn_like(p) * 0.5)
            elif name.endswith("norm.weight"):
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
            elif name.endswith("D"):
                p.copy_(torch.randn_like(p))
    sd = model.state_dict()
    hp = exp.hparams_from_config(cfg)
    g = torch.Generator().manual_seed(seed + 1)
    prompt = torch.randint(0, cfg.vocab_size, (1, prompt_len), generator=g)

    for quant in ("fp16", "int4"):
        entries = exp.collect_tensors(sd, torch.float16, quantize=quant)
        path = HERE / f"{tag}_{quant}.ssm"
        exp.write_ssm(path, hp, entries)
        # Rebuild the exact stored weights in fp32 for the HF run.
        stored = {}
        for e in entries:
            if e.dtype == fmt.DTYPE_INT4_B32:
                stored[e.name] = dequant_int4(e._packed_blob, *e.shape)
            else:
                stored[e.name] = e._tensor.to(torch.float32)
        ref = Mamba2ForCausalLM(cfg).eval()
        ref.load_state_dict(stored, strict=False)
        if "lm_head.weight" in stored:
            ref.lm_head.weight.data.copy_(stored["lm_head.weight"])
        with torch.no_grad():
            out = ref(prompt)
            logits = out.logits[0, -1].float().numpy()
            gen = ref.generate(prompt, max_new_tokens=n_new, do_sample=False,
                               output_scores=True, return_dict_in_generate=True, use_cache=True)
        toks = gen.sequences[0, prompt_len:].numpy().astype(np.uint32)
        step_logits = torch.stack([s[0] for s in gen.scores]).float().numpy()
        np.savez_compressed(HERE / f"{tag}_{quant}_hf.npz", prompt=prompt[0].numpy().astype(np.uint32),
                            prefill_logits=logits, tokens=toks, step_logits=step_logits)


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    args = ap.parse_args()
    fmt, exp = load_reference_tools(args.reference)
    torch.manual_seed(0)
    make_int4_pack(exp)
    make_layout_130m(fmt, exp)
    make_tiny(fmt, exp, "tinyA", dict(d_model=256, n_layer=2, d_state=32, head_dim=32, n_groups=1,
                                      vocab=320, chunk=32), seed=11, prompt_len=45, n_new=8)
    make_tiny(fmt, exp, "tinyB", dict(d_model=128, n_layer=2, d_state=16, head_dim=16, n_groups=4,
                                      vocab=288, chunk=16), seed=12, prompt_len=37, n_new=8)
    print("golden fixtures written to", HERE)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
