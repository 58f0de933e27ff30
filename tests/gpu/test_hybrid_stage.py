"""The tensor-parallel Llama stage (``models.tp_stage``) on one GPU: with one TP rank and every
layer it must compute what ``LlamaModel`` computes with the same weights (same kernels, same
order); and the plan-driven hybrid trainer must train through its public step on one GPU."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _copy_weights(stage, model):
    R, P, M = stage.rep, stage.shd, model.params
    for n in ("embed", "final_norm", "lm_head"):
        M.w(n).copy_(R.w(n))
    for l in model.layer_ids:
        p = f"layers.{l}."
        M.w(p + "attn_norm").copy_(R.w(p + "attn_norm"))
        M.w(p + "mlp_norm").copy_(R.w(p + "mlp_norm"))
        M.w(p + "wqkv").copy_(stage.wqkv(p))
        M.w(p + "wo").copy_(P.w(p + "wo"))
        M.w(p + "w13").copy_(stage.w13(p))
        M.w(p + "w2").copy_(P.w(p + "w2"))


def test_single_rank_stage_matches_llama_model():
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.models.gpt import LlamaModel
    from resihp_megatron_b200.models.tp_stage import TPStage
    from resihp_megatron_b200.parallel.tp_backend import SoloTP

    cfg = TINY.with_(hidden=256, heads=2, kv_heads=1, ffn=512, layers=2, vocab_size=512)  # head dim 128
    S = 256
    stage = TPStage(cfg, "cuda", layers=range(cfg.layers), first=True, last=True, tp=SoloTP("cuda"), micro_batch=1,
                    seq_len=S)
    model = LlamaModel(cfg, "cuda", micro_batch=1, seq_len=S)
    _copy_weights(stage, model)
    g = torch.Generator(device="cuda").manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (S,), device="cuda", generator=g)
    labels = torch.randint(0, cfg.vocab_size, (S,), device="cuda", generator=g)
    stage.forward("mb0", ids_local=ids, labels_local=labels, grad_scale=1.0 / S)
    assert stage.backward("mb0") is None and stage.inflight() == 0
    model.loss_acc.zero_()
    model.forward_backward(ids, labels, 1.0 / S)
    torch.cuda.synchronize()
    a, b = stage.loss_acc.item(), model.loss_acc.item()
    assert math.isfinite(a) and abs(a - b) <= 1e-3 * abs(b), (a, b)
    R, P, M = stage.rep, stage.shd, model.params
    pairs = [(R.g("embed"), M.g("embed")), (R.g("lm_head"), M.g("lm_head")), (R.g("final_norm"), M.g("final_norm"))]
    for l in model.layer_ids:
        p = f"layers.{l}."
        pairs += [(stage.wqkv(p, grad=True), M.g(p + "wqkv")), (P.g(p + "wo"), M.g(p + "wo")),
                  (stage.w13(p, grad=True), M.g(p + "w13")), (P.g(p + "w2"), M.g(p + "w2")),
                  (R.g(p + "attn_norm"), M.g(p + "attn_norm")), (R.g(p + "mlp_norm"), M.g(p + "mlp_norm"))]
    for got, want in pairs:
        err = (got - want).abs().max().item()
        assert err <= 1e-2 * (want.abs().max().item() + 1e-8), err


def test_hybrid_trainer_trains_on_one_gpu():
    import torch.distributed as dist

    from resihp_megatron_b200 import ops
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.train.hybrid_trainer import GPUHybridTrainer, ensure_process_group

    cfg = TINY.with_(hidden=256, heads=2, kv_heads=1, ffn=512, layers=2, vocab_size=512, seq_len=256)
    ensure_process_group(torch.device("cuda", torch.cuda.current_device()))
    try:
        tr = GPUHybridTrainer(cfg, tp=1, pp=1, dp=1, global_batch=4, micro_batch=2, seq_len=256, lr=3e-3)
        l0 = ops.launches()
        losses = [tr.train_step() for _ in range(4)]
        assert ops.launches() > l0
        assert all(math.isfinite(x) for x in losses)
        assert abs(losses[0] - math.log(cfg.vocab_size)) < 0.5  # random init: close to uniform
        assert tr.h2d_bytes_last_step == 2 * 4 * 256 * 8  # ids + labels of the global batch, int64
        tr.close()
    finally:
        dist.destroy_process_group()


def test_single_rank_stage_matches_llama_model_in_fp8_with_gelu():
    """The GPT (GELU) MLP with block-scaled fp8 projections: one TP rank of the stage runs the same
    fp8 kernels in the same order as ``LlamaModel`` -- same loss, gradients and recorded amax."""
    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.models.fp8_linear import Fp8Recipe
    from resihp_megatron_b200.models.gpt import LlamaModel
    from resihp_megatron_b200.models.tp_stage import TPStage
    from resihp_megatron_b200.parallel.tp_backend import SoloTP

    cfg = TINY.with_(hidden=256, heads=2, kv_heads=2, ffn=512, layers=2, vocab_size=512, mlp="gelu")
    S = 256
    stage = TPStage(cfg, "cuda", layers=range(cfg.layers), first=True, last=True, tp=SoloTP("cuda"), micro_batch=1,
                    seq_len=S, fp8=Fp8Recipe())
    model = LlamaModel(cfg, "cuda", micro_batch=1, seq_len=S, fp8=Fp8Recipe())
    R, P, M = stage.rep, stage.shd, model.params
    for n in ("embed", "final_norm", "lm_head"):
        M.w(n).copy_(R.w(n))
    for l in model.layer_ids:
        p = f"layers.{l}."
        for n in ("attn_norm", "mlp_norm"):
            M.w(p + n).copy_(R.w(p + n))
        M.w(p + "wqkv").copy_(stage.wqkv(p))
        M.w(p + "w1").copy_(stage.w13(p))
        M.w(p + "wo").copy_(P.w(p + "wo"))
        M.w(p + "w2").copy_(P.w(p + "w2"))
    g = torch.Generator(device="cuda").manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (S,), device="cuda", generator=g)
    labels = torch.roll(ids, -1)
    stage.forward("mb0", ids_local=ids, labels_local=labels, grad_scale=1.0 / S)
    stage.backward("mb0")
    model.loss_acc.zero_()
    model.forward_backward(ids, labels, 1.0 / S)
    torch.cuda.synchronize()
    a, b = stage.loss_acc.item(), model.loss_acc.item()
    assert math.isfinite(a) and abs(a - b) <= 1e-5 * abs(b), (a, b)
    assert torch.allclose(stage.f8.pending, model.f8.pending, rtol=1e-5, atol=0)
    for l in model.layer_ids:
        p = f"layers.{l}."
        for got, want in ((stage.wqkv(p, grad=True), M.g(p + "wqkv")), (stage.w13(p, grad=True), M.g(p + "w1")),
                          (P.g(p + "wo"), M.g(p + "wo")), (P.g(p + "w2"), M.g(p + "w2"))):
            err = (got - want).abs().max().item()
            assert err <= 1e-5 * (want.abs().max().item() + 1e-12), err


def test_hybrid_trainer_split_backward_matches_1f1b_on_one_gpu():
    """``split_backward=True`` runs each micro-batch's weight-gradient pass as its own W op after
    the input-gradient pass (the zero-bubble order); on one GPU it computes the same sums in the
    same order as plain 1F1B, so the losses agree to bf16 rounding of the deferred GEMMs."""
    import torch.distributed as dist

    from resihp_megatron_b200.models.config import TINY
    from resihp_megatron_b200.train.hybrid_trainer import GPUHybridTrainer, ensure_process_group

    cfg = TINY.with_(hidden=256, heads=2, kv_heads=1, ffn=512, layers=2, vocab_size=512, seq_len=256)
    ensure_process_group(torch.device("cuda", torch.cuda.current_device()))
    try:
        runs = {}
        for name, kw in (("1f1b", {}), ("zb", {"split_backward": True})):
            torch.manual_seed(0)
            tr = GPUHybridTrainer(cfg, tp=1, pp=1, dp=1, global_batch=4, micro_batch=1, seq_len=256, lr=3e-3,
                                  tp_impl="collective", dp_impl="collective", **kw)
            w_ops = sum(ins.op.name == "W" for stream in tr.schedule.values() for ins in stream)
            runs[name] = (w_ops, [tr.train_step() for _ in range(4)])
            tr.close()
        assert runs["1f1b"][0] == 0 and runs["zb"][0] == 4
        for a, b in zip(runs["1f1b"][1], runs["zb"][1]):
            assert math.isfinite(b) and abs(a - b) <= 2e-3 * abs(a), (runs["1f1b"][1], runs["zb"][1])
    finally:
        dist.destroy_process_group()
