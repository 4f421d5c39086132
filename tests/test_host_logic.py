"""Host-side logic that needs no GPU: the install() shim, decay tables, argument
checks and the cache API."""
import math

import pytest
import torch
import torch.nn as nn

import prime_moment_attention_b200 as pma
from prime_moment_attention_b200 import ops


class StandIn(nn.Module):
    """Has the attributes the reference PrimeMomentAttention defines (attention.py:56-75)."""

    def __init__(self):
        super().__init__()
        self.num_heads, self.head_dim, self.num_kv_heads, self.num_kv_groups = 2, 16, 2, 1
        self.decay, self.eps, self.scaling, self.use_qk_norm = 0.99, 1.0, 0.25, False
        self.q_proj = self.k_proj = self.v_proj = self.o_proj = nn.Identity()

    def forward(self, hidden_states, state=None, return_state=False):
        return "original", None


def test_install_uninstall_roundtrip():
    orig = StandIn.__dict__["forward"]
    pma.install(StandIn)
    assert pma.installed(StandIn)
    assert StandIn.forward is pma.moment_forward
    pma.install(StandIn)  # idempotent
    pma.uninstall(StandIn)
    assert StandIn.__dict__["forward"] is orig
    assert StandIn()(torch.zeros(1, 1, 32))[0] == "original"
    pma.uninstall(StandIn)  # no-op


def test_installed_forward_refuses_cpu_tensors():
    pma.install(StandIn)
    try:
        with torch.no_grad(), pytest.raises(RuntimeError, match="CUDA"):
            StandIn()(torch.zeros(1, 4, 32))
    finally:
        pma.uninstall(StandIn)


def test_installed_forward_refuses_autograd():
    m = pma.PrimeMomentAttention(32, 2, 16)
    with pytest.raises(RuntimeError, match="inference-only"):
        m(torch.zeros(1, 4, 32))


def test_lambda_tables():
    t, s = ops.lambda_tensor(0.9, 3, 4, "cpu")
    assert s == 0 and t.shape == (4,) and torch.allclose(t, torch.full((4,), 0.9))
    t, s = ops.lambda_tensor([0.1, 0.2, 0.3, 0.4], 3, 4, "cpu")
    assert s == 0 and t.shape == (4,)
    t, s = ops.lambda_tensor(torch.rand(3, 4), 3, 4, "cpu")
    assert s == 4 and t.shape == (12,)
    with pytest.raises(ValueError):
        ops.lambda_tensor(torch.rand(5), 3, 4, "cpu")


def test_core_rejects_cpu_and_bad_chunk():
    q = torch.zeros(1, 2, 8, 16)
    with pytest.raises(ValueError):
        pma.chunked_prime_ssd_core(q, q, q, chunk_size=0)
    with pytest.raises(RuntimeError, match="CUDA"):
        pma.chunked_prime_ssd_core(q, q, q)


def test_module_constructor_matches_reference_fields():
    m = pma.PrimeMomentAttention(hidden_size=128, num_heads=4, head_dim=32, num_kv_heads=2, decay=0.999,
                                 use_qk_norm=True)
    assert m.num_kv_groups == 2 and m.scaling == 1 / math.sqrt(32) and m.eps == 1.0
    assert m.chunk_size == 64 and m.chunk_threshold == 512
    assert m.k_proj.weight.shape == (64, 128)
    m2 = pma.PrimeMomentAttention(64, 2, 32, decay=[0.9, 0.99])
    assert torch.allclose(m2.decay_per_head, torch.tensor([0.9, 0.99]))
    with pytest.raises(ValueError):
        pma.PrimeMomentAttention(64, 2, 32, decay=[0.9, 0.99, 0.5])


def test_cache_api_matches_reference():
    """Mirrors tests/test_cache.py of the reference."""
    cache = pma.PrimeMomentCache()
    assert cache.get_state(0) is None
    B, H, D = 2, 4, 32
    st = (torch.randn(B, H, D), torch.randn(B, H, D, D), torch.randn(B, H, D, D), torch.randn(B, H, 1),
          torch.randn(B, H, D), torch.randn(B, H, D))
    cache.set_state(layer_idx=0, state=st)
    got = cache.get_state(layer_idx=0)
    assert len(got) == 6 and torch.equal(got[0], st[0])
    cache.update(torch.zeros(B, H, 5, D), torch.zeros(B, H, 5, D), 0)
    cache.update(torch.zeros(B, H, 5, D), torch.zeros(B, H, 5, D), 1)
    assert cache.get_seq_length() == 5
    cache.reset()
    assert cache.get_state(0) is None and cache.get_seq_length() == 0


def test_state_pool_slot_bookkeeping_without_gpu(monkeypatch):
    """Slot allocation, release and row numbering of StatePool (device tensors replaced by CPU)."""
    import torch
    from prime_moment_attention_b200 import ops, pool as P
    real_new = ops.new_state
    monkeypatch.setattr(ops, "new_state", lambda B, H, D, device, zero=True: real_new(B, H, D, "cpu", zero))
    pool = P.StatePool(capacity=4, H=2, D=8, layers=3, device="cpu")
    a, b = pool.alloc(), pool.alloc()
    assert (a, b) == (0, 1) and pool.free_slots == 2
    pool.get_state(2, b)[1].fill_(1.0)
    assert float(pool.state[1][2 * 4 + b].sum()) == 2 * 8 * 8
    assert pool.rows(2, [b, a]).tolist() == [9, 8]
    pool.release(a)
    import pytest
    with pytest.raises(ValueError):
        pool.release(a)
    c = pool.alloc()
    assert c == a
    pool.release(b)
    d = pool.alloc()  # reuse zeroes the slot's rows in every layer
    assert d == b and float(pool.state[1][2 * 4 + b].sum()) == 0.0


def test_module_dtype_cast_keeps_per_head_decay_float32():
    """.to(bfloat16) / .half() cast the projections but not the per-head decays."""
    import torch
    from prime_moment_attention_b200 import attention as A
    m = A.PrimeMomentAttention(64, 2, 32, decay=[0.9995, 0.999]).to(torch.bfloat16)
    assert m.q_proj.weight.dtype == torch.bfloat16
    assert m.decay_per_head.dtype == torch.float32
    assert m.decay_per_head.tolist() == torch.tensor([0.9995, 0.999]).tolist()
    assert m.half().decay_per_head.dtype == torch.float32


class DeltaStandIn(nn.Module):
    """Named like the reference's gated delta-rule module (chunked_delta_prime.py:25)."""

    def _build_features(self, q, k):
        return q, k

    def forward(self, hidden_states, state=None, return_state=False):
        return "original", None


def test_install_picks_the_delta_forward_for_the_delta_module():
    pma.install(DeltaStandIn)
    try:
        assert DeltaStandIn.forward is pma.delta_forward
    finally:
        pma.uninstall(DeltaStandIn)
    assert DeltaStandIn()(torch.zeros(1, 1, 4))[0] == "original"


def test_delta_module_parameters_match_reference_layout():
    """Parameter names and shapes of chunked_delta_prime.py:53-65, gate biases of :67-71."""
    m = pma.ChunkedGatedDeltaPrimeAttention(hidden_size=96, num_heads=4, head_dim=16, num_kv_heads=2)
    shapes = {n: tuple(p.shape) for n, p in m.named_parameters()}
    assert shapes == {"q_proj.weight": (64, 96), "k_proj.weight": (32, 96), "v_proj.weight": (32, 96),
                      "o_proj.weight": (96, 64), "erase_proj.weight": (64, 96), "erase_proj.bias": (64,),
                      "write_proj.weight": (64, 96), "write_proj.bias": (64,), "q_norm.weight": (16,),
                      "q_norm.bias": (16,), "k_norm.weight": (16,), "k_norm.bias": (16,)}
    assert torch.all(m.erase_proj.bias == -2.5) and torch.all(m.write_proj.bias == -1.0)
    assert (m.chunk_size, m.decay, m.lyapunov_bound, m.eps, m.num_kv_groups) == (64, 0.9995, 25.0, 1e-5, 2)


class SelectiveStandIn(nn.Module):
    """Has the selective module's get_tau (selective.py:344-345)."""

    def get_tau(self, device):
        return None

    def forward(self, hidden_states, state=None, return_state=False):
        return "original", None


def test_install_picks_the_selective_forward():
    pma.install(SelectiveStandIn)
    try:
        assert SelectiveStandIn.forward is pma.selective_forward
    finally:
        pma.uninstall(SelectiveStandIn)


def test_selective_module_parameters_and_identity_init():
    """Parameters of selective.py:299-320 and the identity-preserving init of :322-330."""
    m = pma.PrimeSelectiveMomentAttention(hidden_size=64, num_heads=4, head_dim=16, decay=0.99)
    assert {n: tuple(p.shape) for n, p in m.named_parameters()} == {
        "q_proj.weight": (64, 64), "k_proj.weight": (64, 64), "v_proj.weight": (64, 64), "o_proj.weight": (64, 64),
        "q_norm.weight": (16,), "q_norm.bias": (16,), "k_norm.weight": (16,), "k_norm.bias": (16,),
        "delta_proj.weight": (4, 64), "delta_proj.bias": (4,), "log_tau": (4,), "log_beta": (4,)}
    x = torch.randn(2, 5, 64)
    delta = torch.nn.functional.softplus(m.delta_proj(x))
    lam = torch.exp(-delta / m.get_tau(torch.device("cpu")))
    assert torch.allclose(lam, torch.full_like(lam, 0.99), atol=1e-6)
    assert torch.all(m.get_beta(torch.device("cpu")) == 1.0)


def test_new_entries_refuse_cpu_tensors():
    """The fused SwiGLU runs on CUDA tensors only (no CPU fallback); the host-buffer prefill takes
    host tensors and refuses device ones."""
    from prime_moment_attention_b200 import ops
    x = torch.ones(2, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.swiglu(x, x)
    if torch.cuda.is_available():
        q = torch.zeros(1, 1, 4, 64, device="cuda")
        with pytest.raises(ValueError, match="host memory"):
            ops.prefill_from_host(q, q, q, 0.99)
