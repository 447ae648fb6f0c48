"""The persistent decode kernel (one cooperative launch per batch-1 decode
token, ACM_MEGA=1) against the oracle: greedy ids equal the oracle's on every
architecture and weight-type mix of the small models (each mix compiles to a
different kernel instance), and the kernel is the one that ran (its phase
trace can be enabled).  The switch is read once per process, so the check runs
in a child process."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import importlib, json, sys
sys.path.insert(0, {root!r}); sys.path.insert(0, {oracle!r})
acm = importlib.import_module("auto-commit-msg_b200")
synth = importlib.import_module("auto-commit-msg_b200.synth")
import oracle as O
O.build()
out = {{}}
eng = acm.Engine(0)
for name, path in {models!r}.items():
    m = acm.Load(path, 0, engine=eng)
    traced = acm.lib().acm_model_trace(m.handle, 1) == 0
    p = synth.prompt_ids(29, m.Cfg.vocab, 4)
    got = m.Generate(p, acm.Sampler(0.0), 24, stop_on_eos=False)
    want = O.Model(path, 0).generate(p, max_tok=24, stop_on_eos=False)["ids"].tolist()
    out[name] = dict(traced=traced, equal=got == want, got=got, want=want)
    m.close()
eng.close()
print("RESULT " + json.dumps(out))
"""


def test_persistent_decode_matches_oracle(tiny_models):
    models = dict(tiny_models)
    code = CHILD.format(root=ROOT, oracle=os.path.join(ROOT, "oracle"), models=models)
    env = dict(os.environ, ACM_MEGA="1")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    line = next(l for l in r.stdout.splitlines() if l.startswith("RESULT "))
    res = json.loads(line[len("RESULT "):])
    for name, v in res.items():
        assert v["traced"], f"{name}: persistent kernel not in use"
        assert v["equal"], (name, v["got"], v["want"])
