"""Independent cross-check of the oracle against HuggingFace transformers'
own Qwen3 implementation (CPU, fp32, eager attention).

The reference pins nothing numerically at the model level (no golden
vectors, checkpoints absent), so the oracle's block composition — QK-norm,
RoPE, GQA attention, SiLU MLP, tied LM head — is checked against a
third-party Qwen3: the oracle's exactly dequantized weights are loaded into
``Qwen3ForCausalLM`` and the logits compared.  The oracle rounds at the
engine's fp16 precision points and HF does not, so the bound is 5e-3 max abs
on logits of magnitude ~1 (measured ~1.2e-3), and the argmax must agree.

HF rotates half-split pairs (d, d + hd/2).  The engine's default pairwise
RoPE (2p, 2p + 1) is the same model after permuting each head's q/k
projection rows and q/k norm weights (half-split dim p <- 2p,
p + hd/2 <- 2p + 1): attention scores are invariant under a common
permutation of q and k dims and v is untouched.
"""
import numpy as np
import pytest

from oracle import qwen3_ref as R

torch = pytest.importorskip("torch")
transformers = pytest.importorskip("transformers")


def pair_to_half(hd):
    """perm[j] = the pairwise dim that half-split dim j takes."""
    p = np.arange(hd // 2)
    return np.concatenate([2 * p, 2 * p + 1])


def hf_logits(d, cfg, W, toks, rope_style):
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from nnzap_b200 import synth
    hc = Qwen3Config(vocab_size=d.vocab, hidden_size=d.hidden, intermediate_size=d.inter,
                     num_hidden_layers=d.layers, num_attention_heads=d.n_q,
                     num_key_value_heads=d.n_kv, head_dim=d.head_dim, rms_norm_eps=cfg.eps,
                     rope_theta=cfg.rope_theta, tie_word_embeddings=True,
                     max_position_embeddings=256, attn_implementation="eager")
    torch.manual_seed(0)
    m = Qwen3ForCausalLM(hc).float().eval()
    hd = d.head_dim
    perm = pair_to_half(hd) if rope_style == "pairwise" else np.arange(hd)

    def dq(t, M, K):
        return R.dequant_tensor(cfg, t, M, K).astype(np.float32)

    sd = {"model.embed_tokens.weight": dq(W["embed"], d.vocab, d.hidden),
          "model.norm.weight": W["final_norm"]}
    for i, L in enumerate(W["layers"]):
        for key, comp in synth.LAYER_COMPONENTS.items():
            t = L[key]
            if isinstance(t, dict):
                M, K = R.proj_shape(cfg, key)
                w = dq(t, M, K)
                if key in ("q_proj", "k_proj"):
                    heads = M // hd
                    w = w.reshape(heads, hd, K)[:, perm, :].reshape(M, K)
            else:
                w = t[perm] if key in ("q_norm", "k_norm") else t
            sd[f"model.layers.{i}.{comp}.weight"] = np.ascontiguousarray(w)
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = m.load_state_dict({k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in sd.items()},
                                            strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    with torch.no_grad():
        return m(torch.from_numpy(np.asarray(toks))[None]).logits[0].numpy()


@pytest.mark.parametrize("quant,gs", [("q1", 128), ("q4", 64)])
@pytest.mark.parametrize("rope_style", ["pairwise", "half_split"])
def test_oracle_matches_transformers_qwen3(quant, gs, rope_style):
    from nnzap_b200 import synth
    d = synth.ModelDims(vocab=512, hidden=256, inter=512, layers=2, n_q=4, n_kv=2, head_dim=128,
                        gs=gs, quant=quant, rope_style=rope_style)
    W = synth.make_model(d, seed=3)
    cfg = R.Cfg(vocab=d.vocab, hidden=d.hidden, inter=d.inter, layers=d.layers, n_q=d.n_q,
                n_kv=d.n_kv, head_dim=d.head_dim, gs=d.gs, quant=d.quant, rope_style=rope_style)
    toks = np.random.default_rng(1).integers(0, d.vocab, 40)
    ref = R.forward_tokens(cfg, W, toks)
    hf = hf_logits(d, cfg, W, toks, rope_style)
    err = float(np.abs(hf - ref).max())
    assert err <= 5e-3, err
    assert (hf.argmax(1) == ref.argmax(1)).all()
