"""End-to-end numerics of the Llama model on the sm_100a kernels against a PyTorch fp32
autograd implementation of the same architecture and weights."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def torch_reference_loss(model, ids, labels):
    """fp32 autograd Llama forward with the model's own (bf16-rounded) weights."""
    cfg = model.cfg
    P = model.params
    W = {n: P.w(n).float().clone().requires_grad_(True) for n in P.order}
    B, S = model.mb, model.S
    H, D, Hq, Hk = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads
    cos, sin = model.cos, model.sin

    def rms(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.norm_eps) * w

    def rope(x, nh):
        x = x.view(B, S, nh, D)
        c = cos.view(1, S, 1, D // 2).repeat(1, 1, 1, 2)
        s = sin.view(1, S, 1, D // 2).repeat(1, 1, 1, 2)
        rot = torch.cat([-x[..., D // 2:], x[..., : D // 2]], -1)
        return x * c + rot * s

    x = W["embed"][ids.view(-1)]
    for l in model.layer_ids:
        p = f"layers.{l}."
        h = rms(x, W[p + "attn_norm"])
        qkv = h @ W[p + "wqkv"].t()
        q = rope(qkv[:, : Hq * D], Hq).transpose(1, 2)
        k = rope(qkv[:, Hq * D: (Hq + Hk) * D], Hk).transpose(1, 2).repeat_interleave(Hq // Hk, 1)
        v = qkv[:, (Hq + Hk) * D:].view(B, S, Hk, D).transpose(1, 2).repeat_interleave(Hq // Hk, 1)
        att = (q @ k.transpose(-1, -2)) / math.sqrt(D)
        att = att.masked_fill(torch.ones(S, S, device=x.device, dtype=torch.bool).triu(1), float("-inf")).softmax(-1)
        o = (att @ v).transpose(1, 2).reshape(B * S, Hq * D)
        x = x + o @ W[p + "wo"].t()
        h2 = rms(x, W[p + "mlp_norm"])
        gu = h2 @ W[p + "w13"].t()
        F = cfg.ffn
        x = x + (torch.nn.functional.silu(gu[:, :F]) * gu[:, F:]) @ W[p + "w2"].t()
    logits = rms(x, W["final_norm"]) @ W["lm_head"].t()
    loss = torch.nn.functional.cross_entropy(logits, labels.view(-1), reduction="sum")
    return loss, W


def test_llama_step_matches_fp32_reference():
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.models.gpt import LlamaModel

    cfg = TINY.with_(hidden=256, heads=4, kv_heads=2, ffn=512, layers=2, vocab_size=512)
    model = LlamaModel(cfg, "cuda", micro_batch=2, seq_len=128, seed=0)
    g = torch.Generator(device="cuda").manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (2, 128), device="cuda", generator=g)
    labels = torch.randint(0, cfg.vocab_size, (2, 128), device="cuda", generator=g)
    ntok = ids.numel()
    model.loss_acc.zero_()
    model.forward_backward(ids.view(-1), labels.view(-1), grad_scale=1.0 / ntok)
    torch.cuda.synchronize()
    loss = model.loss_acc.item() / ntok
    ref_loss, W = torch_reference_loss(model, ids, labels)
    (ref_loss / ntok).backward()
    assert abs(loss - ref_loss.item() / ntok) < 2e-2 * abs(ref_loss.item() / ntok)
    for name in model.params.order:
        got = model.params.g(name)
        want = W[name].grad
        err = (got - want).abs().max().item()
        scale = want.abs().max().item() + 1e-8
        assert err <= 0.1 * scale, (name, err, scale)


def test_llama_training_reduces_loss_and_is_deterministic():
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.models.gpt import LlamaModel

    cfg = TINY.with_(layers=2)

    def run():
        m = LlamaModel(cfg, "cuda", micro_batch=2, seq_len=128, seed=0)
        g = torch.Generator(device="cuda").manual_seed(3)
        ids = torch.randint(0, cfg.vocab_size, (2, 128), device="cuda", generator=g)
        labels = torch.roll(ids, -1, dims=1)
        out = []
        for _ in range(8):
            m.loss_acc.zero_()
            m.forward_backward(ids.view(-1), labels.view(-1), grad_scale=1.0 / ids.numel())
            m.optimizer_step(lr=3e-3)
            out.append(m.loss_acc.item() / ids.numel())
        return out

    a, b = run(), run()
    assert a == b, "training is not bitwise deterministic"
    assert a[-1] < a[0]


def test_cuda_graph_replay_trains_exactly_like_eager_steps():
    """The whole single-GPU step (micro-batches + Adam, bias corrections read from device memory)
    captured once and replayed: the loss trajectory and the weights equal eager training bit for
    bit (every kernel is deterministic)."""
    from resihp_megatron_b200 import ops
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.train.gpu_trainer import GPUTrainer

    cfg = TINY.with_(layers=2)
    g = torch.Generator().manual_seed(4)
    batches = [torch.randint(0, cfg.vocab_size, (2, 129), generator=g) for _ in range(5)]
    dev = [(b[:, :-1].contiguous().cuda(), b[:, 1:].contiguous().cuda()) for b in batches]

    def run(graph: bool):
        tr = GPUTrainer(cfg, global_batch=2, micro_batch=1, seq_len=128, lr=3e-3, device="cuda")
        losses = []
        for i, (ids, lab) in enumerate(dev):
            if graph and i == 2:
                tr.capture_graphs()
            losses.append(tr.step_device(ids, lab).item())
        return losses, tr.model.params.bf16.clone()

    l0 = ops.launches()
    eager, w_eager = run(False)
    graphed, w_graph = run(True)
    assert ops.launches() > l0
    assert eager == graphed, (eager, graphed)
    assert torch.equal(w_eager, w_graph)


def test_gelu_mlp_step_matches_fp32_reference():
    """GPT MLP (w1 -> gelu -> w2) against PyTorch autograd with the model's weights."""
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.models.gpt import LlamaModel

    cfg = TINY.with_(hidden=256, heads=2, kv_heads=2, ffn=512, layers=2, vocab_size=512, mlp="gelu")
    model = LlamaModel(cfg, "cuda", micro_batch=1, seq_len=128, seed=0)
    g = torch.Generator(device="cuda").manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (1, 128), device="cuda", generator=g)
    labels = torch.roll(ids, -1, 1)
    model.forward_backward(ids.view(-1), labels.view(-1), grad_scale=1.0 / ids.numel())
    torch.cuda.synchronize()
    P = model.params
    W = {n: P.w(n).float().clone().requires_grad_(True) for n in P.order}

    def rms(x, w):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + cfg.norm_eps) * w

    # compare the MLP of layer 0 in isolation: input x2 saved by the model
    x2 = model.x2[0].float()
    h2 = rms(x2, W["layers.0.mlp_norm"])
    out = x2 + torch.nn.functional.gelu(h2 @ W["layers.0.w1"].t(), approximate="tanh") @ W["layers.0.w2"].t()
    assert ((model.xs[1].float() - out).abs().max() / out.abs().max()).item() < 2e-2


def test_fp8_training_tracks_bf16_and_reduces_loss():
    """GPT-style model with block-scaled fp8 linear layers through the trainer: the first loss
    matches the bf16 model's, training reduces it, and the amax history fills one slot per step."""
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.models.fp8_linear import Fp8Recipe
    from resihp_megatron_b200.train.gpu_trainer import GPUTrainer

    cfg = TINY.with_(hidden=256, heads=2, kv_heads=2, ffn=512, layers=2, vocab_size=512, mlp="gelu")
    g = torch.Generator().manual_seed(6)
    data = torch.randint(0, cfg.vocab_size, (2, 129), generator=g)
    ids, lab = data[:, :-1].contiguous().cuda(), data[:, 1:].contiguous().cuda()

    def run(fp8):
        tr = GPUTrainer(cfg, global_batch=2, micro_batch=1, seq_len=128, lr=3e-3, device="cuda",
                        fp8=Fp8Recipe() if fp8 else None)
        return [tr.step_device(ids, lab).item() for _ in range(6)], tr

    bf, _ = run(False)
    f8, tr = run(True)
    assert abs(f8[0] - bf[0]) < 0.02 * bf[0], (f8[0], bf[0])
    assert f8[-1] < f8[0]
    h = tr.model.f8.history
    assert (h[:, :, :6] > 0).all() and (h[:, :, 6:] == 0).all() and not tr.model.f8.has_nonfinite()


def test_fp8_step_replays_as_a_cuda_graph_exactly_like_eager():
    """The fp8 step (weight quantisation, fused norm / activation producers, fp8 GEMMs, amax
    reduction into the history, Adam) allocates nothing and never syncs, so it captures: replays
    train bit for bit like eager steps, and the history keeps one entry per step."""
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.models.fp8_linear import Fp8Recipe
    from resihp_megatron_b200.train.gpu_trainer import GPUTrainer

    cfg = TINY.with_(hidden=256, heads=2, kv_heads=2, ffn=512, layers=2, vocab_size=512, mlp="gelu")
    g = torch.Generator().manual_seed(8)
    batches = [torch.randint(0, cfg.vocab_size, (2, 129), generator=g) for _ in range(5)]
    dev = [(b[:, :-1].contiguous().cuda(), b[:, 1:].contiguous().cuda()) for b in batches]

    def run(graph: bool):
        tr = GPUTrainer(cfg, global_batch=2, micro_batch=1, seq_len=128, lr=3e-3, device="cuda", fp8=Fp8Recipe())
        losses = []
        for i, (ids, lab) in enumerate(dev):
            if graph and i == 2:
                tr.capture_graphs()
            losses.append(tr.step_device(ids, lab).item())
        return losses, tr.model.params.bf16.clone(), tr.model.f8.history.clone()

    eager, w0, h0 = run(False)
    graphed, w1, h1 = run(True)
    assert eager == graphed, (eager, graphed)
    assert torch.equal(w0, w1) and torch.equal(h0, h1)
    assert (h0[:, :, :5] > 0).all() and (h0[:, :, 5:] == 0).all()
