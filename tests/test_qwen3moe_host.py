"""The autograd glue of the patched Qwen3-MoE block (no GPU): the block
workspace keeps the forward's state for the backward, so a model whose decoder
layers recompute their activations in the backward (non-reentrant checkpointing,
as the full-depth setup uses) must produce the same gradients as one that
keeps them.  The device block is replaced by a CPU stand-in with the same
call pattern and the same kind of state (its backward reads what its last
forward stored, not what autograd saved)."""
import pytest
import torch

from usaf_b200 import qwen3moe


class _StandInBlock:
    """forward: y = tanh(hs W_r^T) P, state kept on the object; backward reads it."""

    def __init__(self, E, H, seed):
        g = torch.Generator().manual_seed(seed)
        self.P = torch.randn(E, H, generator=g) * 0.1
        self.state = None
        self.forwards = 0

    def forward(self, hs, w_r, gu, dn):
        self.forwards += 1
        self.state = torch.tanh(hs.float() @ w_r.float().t())
        return (self.state @ self.P).to(hs.dtype)

    def backward(self, dy, hs, w_r, gu, dn):
        t = self.state                                     # the last forward's state
        dl = (dy.float() @ self.P.t()) * (1 - t * t)
        return (dl @ w_r.float()).to(hs.dtype), (dl.t() @ hs.float()).to(w_r.dtype)


class _Dn:
    C = 16


def _grads(recompute: bool, monkeypatch):
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeForCausalLM
    blocks = {}

    def block_for(owner, T, H, E, I, top_k, norm, dtype, device, pair_factor=None):
        key = id(owner)
        if key not in blocks:
            blocks[key] = _StandInBlock(E, H, seed=len(blocks))
        return blocks[key]

    monkeypatch.setattr(qwen3moe, "_block_for", block_for)
    monkeypatch.setattr(qwen3moe, "_int4_of", lambda experts: (None, _Dn()))
    cfg = Qwen3MoeConfig(vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=3,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=8,
                         moe_intermediate_size=16, num_experts=4, num_experts_per_tok=2,
                         norm_topk_prob=True, attention_dropout=0.0)
    torch.manual_seed(0)
    with torch.device("cpu"), qwen3moe.without_dense_experts():
        model = Qwen3MoeForCausalLM(cfg)
    for p in model.parameters():
        p.requires_grad_(False)
    gates = [layer.mlp.gate.weight for layer in model.model.layers]
    for w in gates:
        w.requires_grad_(True)
    if recompute:
        model.gradient_checkpointing_enable(gradient_checkpointing_kwargs={"use_reentrant": False})
    model.train()
    ids = torch.randint(0, 64, (2, 12), generator=torch.Generator().manual_seed(1))
    loss = model(input_ids=ids, labels=ids).loss
    loss.backward()
    return loss.detach(), [w.grad.clone() for w in gates], sum(b.forwards for b in blocks.values())


def test_recompute_gives_the_same_gradients(monkeypatch):
    from transformers.models.qwen3_moe import modeling_qwen3_moe as mq
    orig = (mq.Qwen3MoeSparseMoeBlock.forward, mq.Qwen3MoeExperts.forward)
    qwen3moe.patch_qwen3moe_for_b200()
    try:
        with monkeypatch.context() as m:
            loss_a, grads_a, fwd_a = _grads(False, m)
        with monkeypatch.context() as m:
            loss_b, grads_b, fwd_b = _grads(True, m)
    finally:
        mq.Qwen3MoeSparseMoeBlock.forward, mq.Qwen3MoeExperts.forward = orig
    assert fwd_a == 3 and fwd_b == 6          # recompute ran every block's forward again
    assert torch.equal(loss_a, loss_b)
    for a, b in zip(grads_a, grads_b):
        assert a.abs().sum() > 0
        assert torch.equal(a, b)


def test_blocks_share_backward_scratch_when_configured(monkeypatch):
    """With share_backward, every block of the same sizes gets the same
    backward-only buffers and its own forward state; without it, each block
    allocates its own set."""
    made = []

    class _Scratch:
        def __init__(self, *a):
            self.args = a

    class _Block:
        def __init__(self, dims, device, pair_factor, scratch=None):
            self.scratch, self.pf = scratch, pair_factor
            made.append(self)

    monkeypatch.setattr(qwen3moe, "BackwardScratch", _Scratch)
    monkeypatch.setattr(qwen3moe, "MoEBlock", _Block)
    monkeypatch.setattr(qwen3moe, "_SHARED", {})
    owners = [torch.nn.Module() for _ in range(3)]
    try:
        qwen3moe.configure_workspaces(pair_factor=1.25, share_backward=True)
        blks = [qwen3moe._block_for(o, 64, 32, 4, 16, 2, True, torch.bfloat16, "cpu") for o in owners]
        assert len({id(b) for b in blks}) == 3                      # forward state per layer
        assert len({id(b.scratch) for b in blks}) == 1              # one backward set
        assert blks[0].scratch.args[0] == 64 * 3 and blks[0].pf == 1.25   # ceil(1.25 * 2) pairs/token
        assert qwen3moe._block_for(owners[0], 64, 32, 4, 16, 2, True, torch.bfloat16, "cpu") is blks[0]
        assert qwen3moe.workspaces(torch.nn.ModuleList(owners)) == blks
        qwen3moe.configure_workspaces()
        other = torch.nn.Module()
        b = qwen3moe._block_for(other, 64, 32, 4, 16, 2, True, torch.bfloat16, "cpu")
        assert b.scratch is None and b.pf == 2.0                    # the block allocates its own
    finally:
        qwen3moe.configure_workspaces()


class _Proj:
    def __init__(self, E, R, C, n_ov):
        self.E, self.R, self.C, self.n_ov = E, R, C, n_ov


class _StandInEP:
    """The expert-parallel workspace's call surface: rank 1 of 2, experts 2-3 of 4."""
    rank, El = 1, 2

    def __init__(self, E, H, R, C):
        g = torch.Generator().manual_seed(7)
        self.P = torch.randn(E, H, generator=g) * 0.1
        self.own_cnt = torch.tensor([3, 0], dtype=torch.int32)
        self.R, self.C = R, C
        self.calls = []

    def forward(self, hs, w_r):
        self.state = torch.tanh(hs @ w_r.t())
        return self.state @ self.P

    def backward(self, dy, hs, w_r, reduce_router, compact_gu, compact_dn):
        self.calls.append((reduce_router, compact_gu is not None, compact_dn is not None))
        if compact_gu is not None:
            compact_gu += 1.0
            compact_dn += 2.0
        dl = (dy @ self.P.t()) * (1 - self.state * self.state)
        return dl @ w_r, dl.t() @ hs

    def dense_abs_grad(self, which):
        R, C = (2 * 16, 32) if which == "gate_up_proj" else (32, 16)
        return torch.ones(self.El, R, C)

    def hit_experts(self):
        return (self.own_cnt > 0).nonzero().reshape(-1)

    def expert_candidates(self, which, k):
        return None   # no device gradients here: the store takes the dense |grad| path


def test_expert_parallel_block_glue(monkeypatch):
    """attach(expert_parallel=True) sends the block through the expert-parallel
    workspace: compact gradients of the rank's shard go to its backward, the
    router gradient is summed over ranks, importance captures carry the
    shard's expert offset, and the experts-only entry refuses to run."""
    from transformers.models.qwen3_moe import modeling_qwen3_moe as mq
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from usaf_b200.moe_loader import SparseGradStore, TopKImportanceStore
    orig = (mq.Qwen3MoeSparseMoeBlock.forward, mq.Qwen3MoeExperts.forward)
    qwen3moe.patch_qwen3moe_for_b200()
    try:
        H, I, E = 32, 16, 4
        cfg = Qwen3MoeConfig(vocab_size=64, hidden_size=H, intermediate_size=64, num_hidden_layers=1,
                             num_attention_heads=4, num_key_value_heads=2, head_dim=8,
                             moe_intermediate_size=I, num_experts=E, num_experts_per_tok=2,
                             norm_topk_prob=True)
        with torch.device("cpu"), qwen3moe.without_dense_experts():
            block = mq.Qwen3MoeSparseMoeBlock(cfg)
        gu, dn = _Proj(2, 2 * I, H, 5), _Proj(2, H, I, 3)
        qwen3moe.attach_int4_experts(block.experts, gu, dn, expert_parallel=True)
        ep = _StandInEP(E, H, 2 * I, H)
        monkeypatch.setattr(qwen3moe, "_ep_for", lambda *a: ep)
        monkeypatch.setattr(qwen3moe, "_int4_of", lambda experts: (gu, dn))
        block.gate.weight.requires_grad_(True)
        x = torch.randn(1, 6, H)
        # sparse gradients of the shard
        store = SparseGradStore({"m.gate_up_proj": torch.arange(5), "m.down_proj": torch.arange(3)},
                                {"m.gate_up_proj": (2, 2 * I, H), "m.down_proj": (2, H, I)}, device="cpu")
        block.experts._grad_capture = (store, "m")
        block(x).sum().backward()
        assert ep.calls[-1] == (True, True, True)
        assert torch.equal(store.compact["m.gate_up_proj"], torch.ones(5))
        assert torch.equal(store.compact["m.down_proj"], torch.full((3,), 2.0))
        assert block.gate.weight.grad is not None and block.gate.weight.grad.abs().sum() > 0

        # importance capture: experts numbered in the full tensor (offset rank * El = 2)
        class _Rec(TopKImportanceStore):
            def add_dense_abs(self, name, absg, experts=None, expert_offset=0):
                self.seen = getattr(self, "seen", []) + [(name, tuple(absg.shape), experts.tolist(),
                                                          expert_offset)]

        rec = _Rec({"m.gate_up_proj": (E, 2 * I, H), "m.down_proj": (E, H, I)}, 0.005)
        block.experts._grad_capture = (rec, "m")
        block.gate.weight.grad = None
        block(x).sum().backward()
        assert ep.calls[-1] == (True, False, False)
        assert rec.seen == [("m.gate_up_proj", (2, 2 * I, H), [0], 2), ("m.down_proj", (2, H, I), [0], 2)]
        with pytest.raises(NotImplementedError):
            block.experts(x.reshape(-1, H), torch.ones(6, E))
    finally:
        mq.Qwen3MoeSparseMoeBlock.forward, mq.Qwen3MoeExperts.forward = orig
