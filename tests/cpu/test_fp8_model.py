"""The GPT-style decoder (GELU MLP) with block-scaled fp8 linear layers, run on the CPU through
the kernels' PyTorch emulation (``tests/helpers/fake_kernels``): loss and gradients track the
bf16 model, every recorded amax equals the magnitude of the tensor it stands for, and the
history shifts once per step."""

import pytest
import torch

from resihp_megatron_b200.models.config import GPTConfig

CFG = GPTConfig(name="t-gelu", vocab_size=256, hidden=256, layers=2, heads=2, kv_heads=2, ffn=512, seq_len=128,
                mlp="gelu")


@pytest.fixture
def fakes(monkeypatch):
    from tests.helpers import fake_kernels

    fake_kernels.install(monkeypatch)


def _model(fp8):
    from resihp_megatron_b200.models.fp8_linear import Fp8Recipe
    from resihp_megatron_b200.models.gpt import LlamaModel

    return LlamaModel(CFG, "cpu", micro_batch=1, seq_len=128, seed=3, fp8=Fp8Recipe() if fp8 else None)


def _batch():
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, CFG.vocab_size, (128,), generator=g)
    return ids, torch.roll(ids, -1)


def test_gelu_mlp_parameters():
    from resihp_megatron_b200.models.gpt import layer_param_specs

    names = {s.name.split(".")[-1]: s.shape for s in layer_param_specs(CFG, 0)}
    assert names["w1"] == (512, 256) and "w13" not in names and names["w2"] == (256, 512)
    sharded = {s.name.split(".")[-1] for s in layer_param_specs(CFG, 0, 0, 2)}
    assert "w3" not in sharded and {"w1", "w2"} <= sharded
    assert CFG.layer_params() == 4 * 256 * 256 + 2 * 256 * 512 + 2 * 256


def test_fp8_model_tracks_bf16_and_records_amax(fakes):
    from resihp_megatron_b200.models.fp8_linear import NSLOTS, SLOTS

    ids, labels = _batch()
    ref, m = _model(False), _model(True)
    scale = 1.0 / ids.numel()
    ref.forward_backward(ids, labels, scale)
    m.forward_backward(ids, labels, scale)
    l0, l1 = ref.loss_acc.item(), m.loss_acc.item()
    assert abs(l0 - l1) / abs(l0) < 0.02, (l0, l1)
    for name in m.params.order:
        g0, g1 = ref.params.g(name).flatten(), m.params.g(name).flatten()
        cos = torch.nn.functional.cosine_similarity(g0, g1, dim=0).item()
        assert cos > 0.97, (name, cos)
    # weights' amax: the max |w| of each projection (bf16 copy)
    P = m.params
    for l in range(CFG.layers):
        for lin, wname in (("qkv", "wqkv"), ("o", "wo"), ("fc1", "w1"), ("fc2", "w2")):
            got = m.f8.pending[l, SLOTS[(lin, "w")]].item()
            assert got == P.w(f"layers.{l}.{wname}").float().abs().max().item()
            assert m.f8.pending[l, SLOTS[(lin, "x")]].item() > 0 and m.f8.pending[l, SLOTS[(lin, "dy")]].item() > 0
    # the embedding output is the first layer's residual input, whose rmsnorm feeds qkv
    pend = m.f8.pending.clone()
    m.f8.finish_iteration()
    assert torch.equal(m.f8.history[:, :, 0], pend) and m.f8.pending.abs().sum() == 0
    assert m.f8.history.shape == (CFG.layers, NSLOTS, 16) and not m.f8.has_nonfinite()
    m.f8.finish_iteration()
    assert torch.equal(m.f8.history[:, :, 1], pend) and m.f8.history[:, :, 0].abs().sum() == 0


def test_fp8_weights_requantised_after_each_optimizer_step(fakes):
    ids, labels = _batch()
    m = _model(True)
    m.forward_backward(ids, labels, 1.0 / ids.numel())
    q0 = m.f8.weight(0, "fc1").q_row.float().clone()
    m.optimizer_step(lr=1e-2)
    m.forward_backward(ids, labels, 1.0 / ids.numel())
    q1 = m.f8.weight(0, "fc1").q_row.float()
    assert not torch.equal(q0, q1)
    assert m.f8.version == m.params.step == 1


def test_single_rank_tp_stage_equals_the_model_in_fp8(fakes):
    """``TPStage`` with one TP rank runs the same fp8 operations as ``LlamaModel``."""
    from resihp_megatron_b200.models.fp8_linear import Fp8Recipe
    from resihp_megatron_b200.models.tp_stage import TPStage
    from resihp_megatron_b200.parallel.tp_backend import SoloTP

    ids, labels = _batch()
    m = _model(True)
    st = TPStage(CFG, "cpu", layers=range(CFG.layers), first=True, last=True, tp=SoloTP("cpu"), micro_batch=1,
                 seq_len=128, seed=3, fp8=Fp8Recipe())
    R, P, M = st.rep, st.shd, m.params
    for n in ("embed", "final_norm", "lm_head"):
        R.w(n).copy_(M.w(n))
    for l in range(CFG.layers):
        p = f"layers.{l}."
        for n in ("attn_norm", "mlp_norm"):
            R.w(p + n).copy_(M.w(p + n))
        st.wqkv(p).copy_(M.w(p + "wqkv"))
        st.w13(p).copy_(M.w(p + "w1"))
        P.w(p + "wo").copy_(M.w(p + "wo"))
        P.w(p + "w2").copy_(M.w(p + "w2"))
    m.forward_backward(ids, labels, 1.0 / ids.numel())
    st.forward("mb", ids_local=ids, labels_local=labels, grad_scale=1.0 / ids.numel())
    st.backward("mb")
    assert st.loss_acc.item() == m.loss_acc.item()
    assert torch.equal(st.f8.pending, m.f8.pending)
    for l in range(CFG.layers):
        p = f"layers.{l}."
        assert torch.equal(st.wqkv(p, grad=True), M.g(p + "wqkv"))
        assert torch.equal(st.w13(p, grad=True), M.g(p + "w1"))
        assert torch.equal(P.g(p + "w2"), M.g(p + "w2"))


def test_nonfinite_amax_skips_the_step(fakes):
    """With ``skip_nonfinite`` an iteration whose reduced amax is inf / NaN leaves the weights and
    the optimizer untouched (every rank sees the same reduced amax, so every rank skips)."""
    from resihp_megatron_b200.models.fp8_linear import Fp8Recipe
    from resihp_megatron_b200.train.gpu_trainer import GPUTrainer

    tr = GPUTrainer(CFG, global_batch=1, micro_batch=1, seq_len=128, device="cpu", lr=1e-2,
                    fp8=Fp8Recipe(skip_nonfinite=True))
    ids, labels = _batch()
    ids, labels = ids.view(1, -1), labels.view(1, -1)
    tr.step_device(ids, labels)
    assert getattr(tr, "skipped_steps", 0) == 0 and tr.model.params.step == 1
    P = tr.model.params
    w = P.w("layers.1.w2")
    w[0, 0] = float("inf")  # a diverged weight: its amax (and the step's outputs) are no longer finite
    before = P.master.clone()
    tr.step_device(ids, labels)
    assert tr.skipped_steps == 1 and P.step == 1 and torch.equal(P.master, before)
    assert tr.model.f8.has_nonfinite()


def test_fp8_rejects_shapes_off_the_128_blocks():
    from resihp_megatron_b200.models.fp8_linear import check_shapes

    check_shapes(CFG, 128)
    with pytest.raises(ValueError, match="tokens"):
        check_shapes(CFG, 100)
    with pytest.raises(ValueError, match="ffn"):
        check_shapes(CFG.with_(ffn=640), 128, tp=2)  # 320 per rank
