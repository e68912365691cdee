"""The entropy-gated tree rollout on the B200 path against the reference generator.

``tests/golden/rollout.json`` holds what the reference's ``MentatGenerator``
produced on CPU (``make_golden.py``) for tiny seeded Qwen3 and Llama models in
fp32: every finished or live leaf's generated token ids and log-probability,
the branch points, and the number of decode tokens.  ``TreeRollout`` runs the
same models (identical weights) on the GPU through the paged cache, the
tree-aware decode kernels and the fused gate.  The trees must match exactly:
same leaves, same tokens, same order; log-probabilities to float tolerance.
Each case is run one prompt at a time and with all prompts in lockstep.
"""

import json
import os

import numpy as np
import pytest
import torch

from tests.golden.cases import ROLLOUT_CASES, rollout_model, rollout_prompts

pytestmark = pytest.mark.gpu

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "rollout.json")))


def _rollout(c, model, **kw):
    from mentat_b200.rollout import TreeRollout
    return TreeRollout(model, eos_token_id=c["eos"], max_active_branches=c["max_active_branches"],
                       branching_factor=c["branching_factor"], max_new_tokens=c["max_new_tokens"], block_size=16,
                       max_blocks=4096, **kw)


def _check(name, got, want, tag):
    assert [r["token_ids"] for r in got] == [r["token_ids"] for r in want["results"]], f"{name} {tag}"
    np.testing.assert_allclose([r["log_prob"] for r in got], [r["log_prob"] for r in want["results"]],
                               rtol=1e-4, atol=1e-4, err_msg=f"{name} {tag}")


@pytest.mark.parametrize("name", sorted(ROLLOUT_CASES))
def test_rollout_matches_reference_generator(name):
    c = ROLLOUT_CASES[name]
    model = rollout_model(c, device="cuda")
    prompts = rollout_prompts(c)
    for i, p in enumerate(prompts):
        r = _rollout(c, model)
        got = r.generate(p)
        _check(name, got, GOLDEN[name][i], f"prompt {i}")
        assert r.decode_tokens == GOLDEN[name][i]["decode_tokens_total"]
        assert r.cache.get_stats()["blocks_used"] == 0  # every sequence freed
    # all prompts in lockstep, one forward pass per step
    r = _rollout(c, model)
    for i, got in enumerate(r.generate_many(prompts)):
        _check(name, got, GOLDEN[name][i], f"lockstep prompt {i}")
    assert r.decode_tokens == sum(g["decode_tokens_total"] for g in GOLDEN[name])


@pytest.mark.parametrize("name", sorted(ROLLOUT_CASES))
def test_padded_graphs_match_reference_generator(name):
    """Graphs captured for leaf counts rounded up to a multiple of 4: the padding
    rows append nothing and attend over an empty sequence, and the trees are the
    reference's."""
    c = ROLLOUT_CASES[name]
    model = rollout_model(c, device="cuda")
    r = _rollout(c, model, graph_bucket=4)
    for i, got in enumerate(r.generate_many(rollout_prompts(c))):
        _check(name, got, GOLDEN[name][i], f"padded prompt {i}")
    assert all(n % 4 == 0 for n in r.lm._graphs)
    assert r.cache.get_stats()["blocks_used"] == 0


@pytest.mark.parametrize("name", sorted(ROLLOUT_CASES))
def test_static_decode_matches_reference_generator(name):
    """The eager device-planned step (no graphs) gives the reference's trees too."""
    c = ROLLOUT_CASES[name]
    model = rollout_model(c, device="cuda")
    r = _rollout(c, model, cuda_graphs=False, static_decode=True)
    for i, got in enumerate(r.generate_many(rollout_prompts(c))):
        _check(name, got, GOLDEN[name][i], f"static prompt {i}")


def test_fixed_threshold_extremes():
    """An infinite threshold never branches (one leaf per tree, one token per
    step); a threshold below every entropy branches at the first step, as far
    as the room test M - n >= K allows."""
    import math
    c = ROLLOUT_CASES["qwen3_fp32"]
    model = rollout_model(c, device="cuda")
    prompts = rollout_prompts(c)
    r = _rollout(c, model, entropy_threshold=math.inf)
    res = r.generate_many(prompts)
    assert [len(x) for x in res] == [1] * len(prompts)
    assert all(len(x[0]["token_ids"]) <= c["max_new_tokens"] for x in res)
    r = _rollout(c, model, entropy_threshold=-math.inf)
    res = r.generate_many(prompts)
    assert all(len(x) >= c["branching_factor"] for x in res)
    assert all(len(x) <= c["max_active_branches"] + c["branching_factor"] - 1 for x in res)


def test_calibrated_threshold_is_the_warmup_percentile():
    import numpy as np_
    c = ROLLOUT_CASES["llama_fp32"]
    model = rollout_model(c, device="cuda")
    prompts = rollout_prompts(c)
    r = _rollout(c, model)
    r.entropy_log = []
    keep = r.max_new_tokens
    r.entropy_threshold = float("inf")
    r.max_new_tokens = 9
    r.generate_many(prompts)
    want = float(np_.percentile(np_.asarray(r.entropy_log[len(prompts):]), 75.0))
    r.entropy_log, r.entropy_threshold, r.max_new_tokens = None, None, keep
    thr = r.calibrate_threshold(prompts, steps=8, q=75.0)
    assert thr == want
    assert r.entropy_threshold == thr and r.max_new_tokens == keep and r.decode_tokens == 8 * len(prompts)


def test_graph_workspace_outlives_eager_growth():
    """Captured decode graphs keep writing to the workspace address they were
    captured with.  An eager step that needs a larger workspace must not hand
    the old one back to the allocator: a tensor allocated afterwards must not
    be overwritten by the next replay, and the replayed step must still equal
    the same step run eagerly."""
    from mentat_b200 import PagedKVCacheManager
    from mentat_b200.rollout import PagedLM
    c = ROLLOUT_CASES["qwen3_fp32"]
    model = rollout_model(c, device="cuda")
    prompt = torch.tensor(rollout_prompts(c)[0], device="cuda")

    def setup():
        cache = PagedKVCacheManager(c["layers"], c["kv_heads"], c["head_dim"], max_blocks=512, block_size=16,
                                    device="cuda", dtype=torch.float32)
        lm = PagedLM(model, cache)
        root = cache.allocate_sequence()
        lm.prefill(prompt, root)
        kids = [cache.fork_sequence(root) for _ in range(3)]
        return cache, lm, kids

    tok = lambda n, s: torch.arange(5 + s, 5 + s + n, device="cuda")  # noqa: E731
    cache, lm, kids = setup()
    lm.enable_graphs(max_len=64, max_n=2)
    lm.decode(tok(2, 0), kids[:2])                       # captured (N = 2)
    old = cache._ws.data_ptr()
    lm.decode(tok(3, 1), kids)                           # eager (N = 3 > max_n): a larger workspace
    assert cache._ws.data_ptr() != old
    junk = [torch.full((cache._ws_retired[0].numel(),), 7, dtype=torch.uint8, device="cuda") for _ in range(4)]
    got, _ = lm.decode(tok(2, 2), kids[:2])              # replay of the N = 2 graph
    torch.cuda.synchronize()
    assert all(bool((j == 7).all()) for j in junk)
    cache.check()
    ref_cache, ref_lm, ref_kids = setup()                # the same three steps, eagerly
    ref_lm.decode(tok(2, 0), ref_kids[:2])
    ref_lm.decode(tok(3, 1), ref_kids)
    want, _ = ref_lm.decode(tok(2, 2), ref_kids[:2])
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)
