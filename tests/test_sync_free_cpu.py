"""A training step inside ``sync_free()`` reads no device value on the host.

On CUDA such a read inside a graph capture is an error; here the host-read entry points of
``torch.Tensor`` are patched to raise while the switch is on, and a whole step (forward with
both heads, backward, clip, Muon with a device skip flag, QB commit) runs on the CPU model.
The routed experts use a dense sync-free stand-in for the CPU-only dispatch (the CUDA path
uses the device-routed grouped GEMM).
"""
import pytest
import torch

from kimi_k3_b200 import KimiK3, kimi_k3_cpu_tiny_config
from kimi_k3_b200.runtime import host_checks, sync_free


def _dense_routed(self, latent, ro, accumulation_dtype):
    ex = self.routed_experts
    e = ex.num_experts
    w = torch.zeros(latent.shape[0], e, dtype=accumulation_dtype, device=latent.device)
    w.scatter_add_(1, ro.selected_experts.long(), ro.selected_weights.to(accumulation_dtype))
    g = torch.einsum("ml,ehl->emh", latent, ex.gate_proj)
    u = torch.einsum("ml,ehl->emh", latent, ex.up_proj)
    from kimi_k3_b200.models.primitives import situ_glu_activation
    y = torch.einsum("emh,elh->eml", situ_glu_activation(g, u, ex.beta_gate, ex.beta_up), ex.down_proj)
    return torch.einsum("me,eml->ml", w, y.to(accumulation_dtype))


@pytest.fixture
def host_read_detector(monkeypatch):
    def guard(name):
        orig = getattr(torch.Tensor, name)

        def wrapped(self, *a, **k):
            if not host_checks():
                raise AssertionError(f"host read Tensor.{name} inside sync_free")
            return orig(self, *a, **k)
        monkeypatch.setattr(torch.Tensor, name, wrapped)
    for name in ("__bool__", "item", "tolist", "__int__", "__float__"):
        guard(name)


@pytest.mark.parametrize("qb", ["histogram", "exact"])
def test_training_step_is_sync_free(host_read_detector, monkeypatch, qb):
    import dataclasses
    from kimi_k3_b200.models.moe import StableLatentMoE
    from kimi_k3_b200.train.engine import MoEController, clip_grad_norm_device
    from kimi_k3_b200.train.optimizer import KimiOptimizerConfig, build_kimi_optimizer
    monkeypatch.setattr(StableLatentMoE, "routed_aggregate", _dense_routed)
    cfg = kimi_k3_cpu_tiny_config(enable_vision=False)

    def with_qb(moe_cfg):
        return dataclasses.replace(moe_cfg, quantile_backend=qb)
    cfg = dataclasses.replace(
        cfg, backbone=dataclasses.replace(cfg.backbone, stable_latent_moe_config=with_qb(
            cfg.backbone.stable_latent_moe_config)),
        mtp=dataclasses.replace(cfg.mtp, stable_latent_moe_config=with_qb(cfg.mtp.stable_latent_moe_config)))
    ids = torch.randint(5, 128, (2, 40), generator=torch.Generator().manual_seed(1))
    mask = torch.ones(2, 40, dtype=torch.bool)

    def run(sync_free_mode):
        torch.manual_seed(0)
        model = KimiK3(cfg)
        opt, _ = build_kimi_optimizer(model, KimiOptimizerConfig(muon_lr=0.01))
        ctl = MoEController(model)
        params = [p for p in model.parameters() if p.requires_grad]
        with sync_free(sync_free_mode, all_valid_mask=True):
            ctl.begin()
            out = model(input_ids=ids, attention_mask=mask, labels=ids, use_mtp=True, compute_logits=False)
            out.loss.backward()
            gnorm = clip_grad_norm_device(params, 1.0)
            if sync_free_mode:
                found_inf = ~torch.isfinite(gnorm)
                opt.muon.step(skip=found_inf)
                ctl.commit(keep_old=found_inf)
            else:
                opt.muon.step()
                ctl.commit()
        return model, out.loss.detach()

    eager, l1 = run(False)
    device, l2 = run(True)
    assert torch.equal(l1, l2)
    for (n, a), (_, b) in zip(eager.state_dict().items(), device.state_dict().items()):
        assert torch.allclose(a, b, rtol=0, atol=1e-6), n
