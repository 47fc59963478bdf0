"""CPU: the Mamba model wrapper's configuration and weight mapping (no compute)."""
import math
import warnings

import pytest
import torch

from mamba_onnx.model import MambaConfig, MambaLM, mamba_130m


def _hf_model(cfg: MambaConfig, seed: int = 0):
    transformers = pytest.importorskip("transformers")
    torch.manual_seed(seed)
    hf_cfg = transformers.MambaConfig(vocab_size=cfg.vocab_size, hidden_size=cfg.d_model,
                                      state_size=cfg.d_state, num_hidden_layers=cfg.n_layer,
                                      expand=cfg.expand, conv_kernel=cfg.d_conv,
                                      layer_norm_epsilon=cfg.rms_eps)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        return transformers.MambaForCausalLM(hf_cfg)


def test_mamba_130m_shape():
    cfg = mamba_130m()
    assert (cfg.d_model, cfg.n_layer, cfg.d_inner, cfg.d_state, cfg.rank, cfg.d_conv) == \
        (768, 24, 1536, 16, 48, 4)
    model = MambaLM(cfg)
    n = sum(p.numel() for p in model.parameters())
    assert 129e6 < n < 130e6  # tied embeddings: 129.1 M


def test_parameter_count_matches_transformers():
    cfg = MambaConfig(d_model=64, n_layer=3, vocab_size=100)
    hf = _hf_model(cfg)
    ours = MambaLM(cfg)
    # the HF count includes the tied lm_head once
    assert sum(p.numel() for p in ours.parameters()) == sum(p.numel() for p in hf.parameters())


def test_load_hf_state_dict_copies_every_tensor():
    cfg = MambaConfig(d_model=64, n_layer=2, vocab_size=100)
    hf = _hf_model(cfg, seed=3)
    sd = hf.state_dict()
    ours = MambaLM(cfg).load_hf_state_dict(sd)
    assert torch.equal(ours.embedding, sd["backbone.embeddings.weight"])
    assert torch.equal(ours.norm_f_weight, sd["backbone.norm_f.weight"])
    for i, layer in enumerate(ours.layers):
        for name, hf_name in MambaLM.HF_NAMES.items():
            assert torch.equal(getattr(layer, name), sd[f"backbone.layers.{i}.{hf_name}"]), name
    # every layer tensor of the HF model is mapped
    mapped = {f"backbone.layers.{i}.{n}" for i in range(cfg.n_layer) for n in MambaLM.HF_NAMES.values()}
    layer_keys = {k for k in sd if k.startswith("backbone.layers.")}
    assert layer_keys == mapped


def test_init_random_follows_mamba_init():
    cfg = MambaConfig(d_model=64, n_layer=2, vocab_size=100)
    m = MambaLM(cfg).init_random(seed=5)
    for layer in m.layers:
        assert torch.allclose(layer.A_log, torch.log(torch.arange(1, 17.0)).repeat(cfg.d_inner, 1))
        dt = torch.nn.functional.softplus(layer.dt_proj_bias)
        assert dt.min() >= 1e-3 * (1 - 1e-5) and dt.max() <= 1e-1 * (1 + 1e-5)
        assert torch.all(layer.D == 1) and torch.all(layer.conv_bias == 0)
        assert abs(layer.in_proj_weight.std().item() - 0.02) < 0.002
    # deterministic in the seed
    m2 = MambaLM(cfg).init_random(seed=5)
    assert all(torch.equal(a, b) for a, b in zip(m.parameters(), m2.parameters()))
    assert math.isclose(cfg.rank, 4)
