"""Host-side checks that need no GPU: the C-ABI library builds for sm_100a,
loads, and exports every symbol include/qb.h declares; argument validation
fails with the right status before any launch; configs, weight packing,
checkpoints and the stream_decode ordering behave."""
import os
import re
from types import SimpleNamespace

import pytest
import torch

from conftest import ROOT


def _declared_symbols():
    with open(os.path.join(ROOT, "include", "qb.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(qb_[a-z0-9_]+)\s*\(", text)))


def test_header_symbols_are_exported(built_lib):
    from hackthenorth_b200 import _lib

    names = _declared_symbols()
    assert "qb_decode_step" in names and "qb_grouped_attention" in names
    for n in names:
        assert hasattr(built_lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"


def test_library_is_built_for_sm100a(built_lib):
    from hackthenorth_b200 import _lib

    assert b"sm_100a" in built_lib.qb_version()
    with open(_lib.LIB_PATH, "rb") as f:
        blob = f.read()
    assert b"sm_100a" in blob


def test_argument_validation_without_launch(built_lib):
    from hackthenorth_b200 import _lib

    L = built_lib
    # NULL pointers and bad shapes are rejected on the host with QB_ERR_ARG.
    assert L.qb_norm_projection(None, None, None, None, 256, 4, 1e-6, 0, None) == _lib.QB_ERR_ARG
    assert b"16-byte" in L.qb_last_error(None)
    assert L.qb_projection_residual(16, 16, 16, 16, 100, 4, None) == _lib.QB_ERR_UNSUPPORTED
    cfg = _lib.QbConfig(1024, 16, 8, 64, 3072, 28, 151936, 1e-6)
    ctx = _lib.c_void_p()
    assert L.qb_create(_lib.ctypes.byref(cfg), 0, 0, 1, _lib.ctypes.byref(ctx)) == _lib.QB_ERR_UNSUPPORTED
    cfg = _lib.QbConfig(1000, 16, 8, 128, 3072, 28, 151936, 1e-6)
    assert L.qb_create(_lib.ctypes.byref(cfg), 0, 0, 1, _lib.ctypes.byref(ctx)) == _lib.QB_ERR_UNSUPPORTED
    with pytest.raises(ValueError):
        _lib.check(_lib.QB_ERR_ARG)


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from hackthenorth_b200 import _lib

    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU or PyTorch fallback"):
        _lib.load()


def test_configs_and_bytes():
    from hackthenorth_b200.config import QWEN3_0P6B, QWEN3_4B, QWEN3_8B, ModelConfig

    # per-token weight bytes quoted for the three shapes (norm gains included)
    assert abs(QWEN3_4B.weight_bytes_per_token() - 8_044_544_000) < 2_000_000
    assert abs(QWEN3_8B.weight_bytes_per_token() - 15_136_194_560) < 2_000_000
    assert abs(QWEN3_0P6B.weight_bytes_per_token() - 1_191_968_768) < 2_000_000
    assert QWEN3_8B.kv_bytes_per_context_token() == 147_456
    assert QWEN3_0P6B.kv_bytes_per_context_token() == 114_688
    rt = ModelConfig.from_hf(QWEN3_4B.to_hf(), name="x")
    assert rt.hidden == 2560 and rt.rope_theta == 5e6 and rt.tied


def test_gate_up_interleave_and_checkpoint_roundtrip(tmp_path):
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.weights import interleave_gate_up, load_checkpoint, random_state_dict, save_checkpoint

    g = torch.arange(12, dtype=torch.float32).reshape(3, 4)
    u = -g
    gu = interleave_gate_up(g, u)
    assert torch.equal(gu[0], g[0]) and torch.equal(gu[1], u[0]) and torch.equal(gu[5], u[2])
    state = random_state_dict(QWEN3_SMALL, 0)
    again = random_state_dict(QWEN3_SMALL, 0)
    assert all(torch.equal(state[k], again[k]) for k in state)
    w = state["model.layers.0.self_attn.q_proj.weight"].float()
    assert 0.018 < w.std().item() < 0.022
    save_checkpoint(str(tmp_path), QWEN3_SMALL, state)
    cfg, loaded = load_checkpoint(str(tmp_path))
    assert cfg.hidden == QWEN3_SMALL.hidden and cfg.vocab == QWEN3_SMALL.vocab
    assert all(torch.equal(state[k], loaded[k]) for k in state)


@pytest.mark.parametrize("depth", [1, 2, 3])
def test_stream_decode_launches_before_yield_without_extra_steps(depth):
    # dryft/tests/test_decode.py:20-38; depth > 1: a token ring keeps that many
    # replays ahead of the consumer, tokens still in order, no extra replays
    from hackthenorth_b200.engine import stream_decode

    class Handle:
        def __init__(self, value):
            self.value = value

        def result(self):
            return [self.value]

    for length in (1, 2, 5, 9):
        token = [0]
        launches = []

        def step():
            token[0] += 1
            launches.append(1)

        state = SimpleNamespace(step=step, read_token=lambda: list(token))
        if depth > 1:
            state.read_token_async = lambda slots: Handle(token[0])
        saved = []
        for i, out in enumerate(stream_decode(state, [0], length, depth=depth)):
            assert out == [i]
            assert len(launches) == min(i + depth, length - 1)
            saved.append(out)
        assert len(launches) == length - 1 and len(saved) == length
