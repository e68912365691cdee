"""Runs the reference's own ``MentatGenerator`` on a CUDA device, in a process of
its own, and writes its trees as JSON (used by ``tests/test_gpu_dropin.py``).

    python tests/dropin_child.py {mentat|reference} OUT.json CASE[:DTYPE] ...

The reference is the pip-installed copy under ``baseline/_ref``.

* ``mentat``: before the reference is imported, the module aliases of the
  integration guide are installed: ``core.paged_kv_cache.PagedKVCacheManager``
  is this package's cache manager and ``adapters.attention_backend`` is
  ``mentat_b200.attention_backend``.  The reference's adapters then call this
  package's ``build_packed_kv`` and ``attn_decode`` unchanged.
* ``reference``: the reference as it ships (its paged cache, its attention
  backend: flash-attn when it loads, else its SDPA path).

Every decode step's active leaves (their generated token ids) are recorded by
wrapping the generator's batched forward, so the trees can be compared step by
step.
"""

from __future__ import annotations

import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
sys.path.insert(0, ROOT)
sys.path.insert(1, REF)

import torch  # noqa: E402


class StubTokenizer:
    """The generator's tokenizer interface over space-separated token ids."""

    def __init__(self, eos):
        self.eos_token_id = eos

    def __call__(self, prompt, return_tensors="pt"):
        return {"input_ids": torch.tensor([[int(t) for t in prompt.split()]], dtype=torch.long)}

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(int(t)) for t in ids)


def main():
    mode, out_path, cases = sys.argv[1], sys.argv[2], sys.argv[3:]
    backend = None
    if mode == "mentat":
        import mentat_b200
        import mentat_b200.attention_backend as mab
        import core.paged_kv_cache as pk
        pk.PagedKVCacheManager = mentat_b200.PagedKVCacheManager   # generator.py builds it (:92-100)
        sys.modules["adapters.attention_backend"] = mab             # the adapters import attn_* from here
        backend = mab.BACKEND
    else:
        import adapters.attention_backend as ab
        if ab.BACKEND == "flash":
            try:  # flash-attn may have no kernels for this GPU: then the reference's own SDPA path
                q = torch.zeros((1, 16, 2, 64), device="cuda", dtype=torch.bfloat16)
                ab.flash_attn_func(q, q, q, causal=True)
                torch.cuda.synchronize()
            except Exception:
                ab.BACKEND = "sdpa"
        backend = ab.BACKEND
    import core.generator_utils as gu
    from core.generator import MentatGenerator
    from tests.golden.cases import ROLLOUT_CASES, rollout_model, rollout_prompts, sharpen

    trees = {"backend": backend, "cases": {}}
    for spec in cases:
        name, _, dt = spec.partition(":")
        c = ROLLOUT_CASES[name]
        dtype = {"": torch.float32, "f32": torch.float32, "bf16": torch.bfloat16}[dt]
        model = rollout_model(c, device="cuda").to(dtype)
        if dt == "bf16":
            model = sharpen(model)
        runs = []
        for prompt in rollout_prompts(c):
            gen = MentatGenerator(model, StubTokenizer(c["eos"]), max_active_branches=c["max_active_branches"],
                                  branching_factor=c["branching_factor"], max_new_tokens=c["max_new_tokens"],
                                  block_size=16, max_blocks=2048)
            steps = []
            trees_seen = []
            init = gu.PrefixTree.__init__

            def tree_init(self, *a, **kw):
                init(self, *a, **kw)
                trees_seen.append(self)

            decode = gen.wrapper.decode_batch

            def decode_batch(token_ids, seq_ids, *a, **kw):
                steps.append(sorted(leaf.get_full_sequence() for leaf in trees_seen[-1].get_active_leaves()))
                return decode(token_ids, seq_ids, *a, **kw)

            gu.PrefixTree.__init__ = tree_init
            gen.wrapper.decode_batch = decode_batch
            try:
                res = gen.generate(" ".join(map(str, prompt)))
            finally:
                gu.PrefixTree.__init__ = init
            d = gen.get_diagnostics()
            runs.append({"results": [{"token_ids": r["token_ids"], "log_prob": r["log_prob"]} for r in res],
                         "steps": steps, "decode_tokens_total": d["decode_tokens_total"]})
        trees["cases"][spec] = runs
    with open(out_path, "w") as f:
        json.dump(trees, f)


if __name__ == "__main__":
    main()
