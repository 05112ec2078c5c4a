"""Launch chunks replayed as CUDA graphs give the same embeddings as direct launches.

The library captures each launch-chunk shape into a CUDA graph on its first use and replays
it afterwards (GLP_GRAPHS=0 turns this off).  The tests run the small conditioned model with
and without graphs in child processes (the switch is read once per process) and compare
bit for bit, over repeated calls (replays) and two interleaved shapes, and check that the
library's launch counters keep counting replayed launches.
"""
from __future__ import annotations

import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = textwrap.dedent("""
    import sys, numpy as np
    from glypr_b200 import api, synth
    path, out = sys.argv[1], sys.argv[2]
    res = {}
    with api.GlyprEmbedder.load_gguf(path, [0]) as emb:
        a_ids, a_lens = synth.make_batch(3, 512, emb.info.vocab, lengths=[512, 200, 31])
        b_ids, b_lens = synth.make_batch(1, 700, emb.info.vocab, seed=5, lengths=[700])
        emb.profile_read()  # reset the counters
        for i in range(3):
            res[f"a{i}"] = emb.embed_tokens(a_ids, a_lens)
            res[f"launches_a{i}"] = np.array(emb.profile_read()["_total_launches"])
            res[f"b{i}"] = emb.embed_tokens(b_ids, b_lens, out_dim=256)
            res[f"launches_b{i}"] = np.array(emb.profile_read()["_total_launches"])
    np.savez(out, **res)
""")


def _run(path, out, graphs):
    env = dict(os.environ)
    env.pop("GLP_GRAPHS", None)
    if not graphs:
        env["GLP_GRAPHS"] = "0"
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    r = subprocess.run([sys.executable, "-c", SCRIPT, path, out], env=env, cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    return np.load(out)


def test_graph_replays_match_direct_launches(small_cond_gguf, tmp_path):
    direct = _run(small_cond_gguf, str(tmp_path / "direct.npz"), graphs=False)
    graphs = _run(small_cond_gguf, str(tmp_path / "graphs.npz"), graphs=True)
    for i in range(3):
        for k in ("a", "b"):
            np.testing.assert_array_equal(graphs[f"{k}{i}"], direct[f"{k}0"])
            np.testing.assert_array_equal(direct[f"{k}{i}"], direct[f"{k}0"])
            # replays count the same launches as the captured (and the direct) run
            assert int(graphs[f"launches_{k}{i}"]) == int(direct[f"launches_{k}0"]) > 0
