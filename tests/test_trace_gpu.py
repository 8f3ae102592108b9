"""Step tracing (qb_set_trace / hackthenorth_b200.trace): every launch of a
captured decode step records its CTAs' timestamps, the labels name the
launches in order, the stamps are ordered, and a traced step computes the
same tokens as an untraced one."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_trace_records_every_launch_of_a_step(built_lib):
    from hackthenorth_b200.config import QWEN3_SMALL
    from hackthenorth_b200.engine import Engine
    from hackthenorth_b200.trace import ENTRY, EXIT, WAIT, StepTrace

    cfg = QWEN3_SMALL
    engine = Engine.from_random(cfg, seed=0)
    prompt = list(range(5, 21))
    st = engine.new_state(len(prompt), 8, keep_logits=True)
    st.prefill(torch.tensor(prompt, device=engine.device))
    first = st.read_token()[0]
    plain = []
    for _ in range(3):
        st.step()
        plain += st.read_token()
    st.check()

    st.prefill(torch.tensor(prompt, device=engine.device))
    tr = StepTrace(st)
    traced = []
    for _ in range(3):
        st.step()
        traced += st.read_token()
    st.check()
    assert st.read_token() != [] and traced == plain and first is not None

    labels = tr.labels()
    want = [f"{k} {l}" for l in range(cfg.n_layers) for k in ("qkv", "attn", "o", "gateup", "down")]
    assert labels == want + [f"head {cfg.n_layers}"]
    for rec in tr.launches():
        s = rec["stamps"]
        assert len(s) > 0, rec["label"]
        assert bool((s[:, EXIT] >= s[:, ENTRY]).all())
        w = s[:, WAIT] > 0
        assert bool((s[w, WAIT] >= s[w, ENTRY]).all()) and bool((s[w, EXIT] >= s[w, WAIT]).all())
    summ = tr.summary()
    assert len(summ["launches"]) == len(labels)
    spans = sum(r["span"] for r in summ["launches"])
    assert abs(spans - summ["step_us"]) <= 0.05 * summ["step_us"] + 1.0
    assert 0 < summ["step_us"] < 10000
    tr.close()
    st.step()  # recaptured without tracing
    st.check()
