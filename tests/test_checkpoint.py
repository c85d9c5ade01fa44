"""Checkpoint layout (reference trainer keys) and resume: a resumed run continues bit-exactly."""
import copy

import torch
import torch.nn as nn

from my_muon_fsdp2_b200 import FSDPMuonOptimizer, MuonOptimizer
from my_muon_fsdp2_b200.train import load_checkpoint, save_checkpoint


def _setup():
    torch.manual_seed(0)
    m = nn.Sequential(nn.Linear(16, 32), nn.GELU(), nn.Linear(32, 8))
    return m


def _step(m, opt, s):
    torch.manual_seed(100 + s)
    x, y = torch.randn(4, 16), torch.randn(4, 8)
    opt.zero_grad()
    loss = ((m(x) - y) ** 2).mean()
    loss.backward()
    opt.step()
    return loss.item()


def test_save_resume_bit_exact(tmp_path):
    m = _setup()
    opt = FSDPMuonOptimizer(m, lr=0.02)
    for s in range(2):
        loss = _step(m, opt, s)
    path = save_checkpoint(str(tmp_path), "mlp", m, opt, epoch=1, loss=loss)
    ck = torch.load(path, weights_only=False)
    assert set(ck) == {"model_state_dict", "optimizer_state_dict", "epoch", "loss"}
    assert ck["optimizer_state_dict"]["step_count"] == 2
    assert set(next(iter(ck["optimizer_state_dict"]["state"].values()))) == {"momentum_buffer", "second_moment",
                                                                             "accum_count"}
    cont = [_step(m, opt, s) for s in range(2, 4)]
    m2 = _setup()
    opt2 = FSDPMuonOptimizer(m2, lr=0.02)
    info = load_checkpoint(path, m2, opt2)
    assert info["epoch"] == 1 and opt2._step_count == 2
    cont2 = [_step(m2, opt2, s) for s in range(2, 4)]
    assert cont == cont2
    for p, q in zip(m.parameters(), m2.parameters()):
        assert torch.equal(p, q)


def test_two_optimizers(tmp_path):
    m = _setup()
    opts = [MuonOptimizer([m[0].weight, m[2].weight]), torch.optim.AdamW([m[0].bias, m[2].bias])]
    path = save_checkpoint(str(tmp_path), "two", m, opts, epoch=0, loss=0.0)
    m2 = _setup()
    opts2 = [MuonOptimizer([m2[0].weight, m2[2].weight]), torch.optim.AdamW([m2[0].bias, m2[2].bias])]
    load_checkpoint(path, m2, opts2)


def test_trainer_clips_gradient_norm():
    """max_grad_norm (the reference trainers clip at 1.0): gradients leave the step with global
    norm <= the bound, and the pre-clip norm is reported."""
    import torch.nn as nn

    from my_muon_fsdp2_b200.train import Trainer

    class Toy(nn.Module):
        def __init__(self):
            super().__init__()
            self.emb = nn.Embedding(16, 8)
            self.out = nn.Linear(8, 16)

        def forward(self, x, y):
            return 100.0 * nn.functional.cross_entropy(self.out(self.emb(x)).flatten(0, 1), y.flatten())

    torch.manual_seed(0)
    model = Toy()
    seen = {}

    class Probe(torch.optim.SGD):
        def step(self, closure=None):
            seen["norm"] = torch.sqrt(sum((p.grad.float() ** 2).sum() for p in model.parameters()))
            return super().step(closure)

    trainer = Trainer(model, [Probe(model.parameters(), lr=0.0)], grad_accum=2, device="cpu", max_grad_norm=1.0)
    batch = torch.randint(0, 16, (2, 3, 9))
    trainer.train_step(batch)
    assert float(trainer.last_grad_norm) > 1.0
    assert float(seen["norm"]) <= 1.0 + 1e-4
    m = trainer.last_metrics
    assert m["step"] == 1 and m["micro_batches"] == 2 and m["tokens"] == 2 * 3 * 8
    assert float(m["grad_norm"]) == float(trainer.last_grad_norm)
    s = trainer.metrics_summary()  # device values read back; no step timing on CPU
    assert isinstance(s["loss"], float) and s["grad_norm"] == float(trainer.last_grad_norm)
    assert "step_ms" not in s and trainer.last_step_ms() is None
