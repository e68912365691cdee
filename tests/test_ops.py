"""The torch operators the public API calls: schemas and fake implementations (CPU).

``attn_decode``, ``append_tokens_batched`` and ``Gate.launch`` reach the C ABI
through ``torch.ops.mentat_b200.*``.  Here each operator is checked for its
registered schema and, under FakeTensorMode, for the output its fake
implementation reports, which is what torch.compile traces with.  No library
call is made.
"""

import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import mentat_b200  # noqa: F401  (registers the operators)
import mentat_b200.attention_backend  # noqa: F401
import mentat_b200.gate  # noqa: F401


def test_schemas():
    s = str(torch.ops.mentat_b200.paged_decode.default._schema)
    assert s.startswith("mentat_b200::paged_decode(Tensor q, Tensor slots,") and s.endswith("-> Tensor")
    s = str(torch.ops.mentat_b200.append_batched.default._schema)
    assert "Tensor(a0!) k_pool" in s and "Tensor(a1!) v_pool" in s and s.endswith("-> ()")
    s = str(torch.ops.mentat_b200.gate_step.default._schema)
    assert "float[] params" in s and "Tensor(a6!) out" in s and s.endswith("-> ()")


def test_fake_implementations():
    with FakeTensorMode():
        q = torch.empty(64, 32, 128, dtype=torch.bfloat16)
        slots = torch.empty(64, dtype=torch.int32)
        out = torch.ops.mentat_b200.paged_decode(q, slots, 4096, 1, 0, 0.088)
        assert out.shape == q.shape and out.dtype == q.dtype
        pool = torch.empty(2, 16, 8, 128, dtype=torch.bfloat16)
        kv = torch.empty(64, 8, 128, dtype=torch.bfloat16)
        assert torch.ops.mentat_b200.append_batched(pool, pool, slots, kv, kv, 1, 0) is None
        logits = torch.empty(4, 1000, dtype=torch.bfloat16)
        i32 = torch.empty(5, dtype=torch.int32)
        f64 = torch.empty(4, dtype=torch.float64)
        rec = torch.empty(4 * 128, dtype=torch.uint8)
        assert torch.ops.mentat_b200.gate_step(logits, i32, i32, f64, [0.7, 1.2, 0.3, 1.25, 0.3],
                                               [3, 10, 4, 0, 10], rec) is None
