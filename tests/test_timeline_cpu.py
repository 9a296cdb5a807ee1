"""The phase-timeline summary (infernt_b200.timeline.summarize) on a
synthetic trace with known marks: 2 layers (11 phases), 3 steps, 4 CTAs."""
import numpy as np

from infernt_b200 import timeline as T


def make_trace(num_layers=2, steps=3, ctas=4):
    P = 5 * num_layers + 1
    tr = np.zeros((ctas, steps, P, 9), dtype=np.int64)
    t = 1_000_000
    for s in range(steps):
        for p in range(P):
            kind = "lm_head" if p == P - 1 else T.KINDS[p % 5]
            for c in range(ctas):
                f = tr[c, s, p]
                f[0] = t
                if kind == "attention":
                    if c == 0:  # one CTA owns the only item
                        f[1], f[7], f[8], f[4], f[2] = t + 500, t + 700, t + 900, t + 1500, t + 3000
                    else:
                        f[2] = t + 100
                else:
                    f[7] = t + 1000           # inputs current 1 us after the previous phase
                    f[1] = t + 1200
                    f[2] = t + 1200 + 2000 + 100 * c  # work 2.0-2.3 us; CTA 3 last
                    f[4] = t + 800             # producer done before the inputs
                    f[5] = 1965                # 1 us of consumer wait at 1965 MHz
                f[3] = f[2]
            t = int(tr[:, s, p, 2].max())
    return tr


def test_summary_of_known_marks():
    tr = make_trace()
    s = T.summarize(tr, 2)
    q = s["qkv"]
    assert abs(q["crit"] - 3.5) < 1e-9      # 1.2 + 2.0 + 0.3 us after the previous phase's last CTA
    assert abs(q["inputs"] - 1.0) < 1e-9
    assert abs(q["work"] - 2.15) < 1e-9     # median of 2.0, 2.1, 2.2, 2.3
    assert abs(q["spread"] - 0.15) < 1e-9   # 3.5 - median(3.2, 3.3, 3.4, 3.5)
    assert abs(q["cwait"] - 1.0) < 1e-9
    assert abs(q["issued"] - 0.8) < 1e-9
    a = s["attention"]
    assert a["items"] == 1.0
    assert abs(a["crit"] - 3.0) < 1e-9 and abs(a["landed"] - 0.5) < 1e-9
    assert abs(a["partial_last"] - 1.5) < 1e-9
    # every phase takes 3.5 us except attention (3.0): 2 layers x 17 + LM head 3.5
    assert abs(s["step_us"] - (2 * (4 * 3.5 + 3.0) + 3.5)) < 1e-9
    text = T.format_summary(s, 2)
    assert "layer critical path 17.00 us x 2 layers" in text


def test_cli_summarises_a_saved_trace(tmp_path, capsys):
    # a TinyLlama-shaped trace (22 layers, 111 phases) through the --load path
    tr = make_trace(num_layers=22, steps=2, ctas=3)
    path = tmp_path / "trace.npy"
    np.save(path, tr)
    assert T.main(["--load", str(path), "--shape", "tinyllama"]) == 0
    out = capsys.readouterr().out
    assert "| qkv | 3.40 | 1.00 |" in out  # 1.2 + 2.2 us: the third CTA is the last
    assert "x 22 layers" in out
