"""The rf-detr patch registry, exercised against stub modules (rf-detr is not installed here)."""

import sys
import types

import pytest
import torch

from rfdetr_training_throughput_b200 import matcher, patches


@pytest.fixture()
def fake_rfdetr(monkeypatch):
    class HungarianMatcher:
        def __init__(self):
            self.cost_class, self.cost_bbox, self.cost_giou, self.focal_alpha = 2.0, 5.0, 2.0, 0.25

        def _compute_compact_detection_cost_matrix(self, outputs, targets, *, clamp_target_labels=False):
            return "upstream"

        def forward(self, outputs, targets, group_detr=1):
            return "upstream"

    mods = {
        "rfdetr": types.ModuleType("rfdetr"),
        "rfdetr.models": types.ModuleType("rfdetr.models"),
        "rfdetr.models.matcher": types.ModuleType("rfdetr.models.matcher"),
        "rfdetr.models._assignment": types.ModuleType("rfdetr.models._assignment"),
        "rfdetr.models.criterion": types.ModuleType("rfdetr.models.criterion"),
        "rfdetr.models.ops": types.ModuleType("rfdetr.models.ops"),
        "rfdetr.models.ops.modules": types.ModuleType("rfdetr.models.ops.modules"),
        "rfdetr.models.ops.modules.ms_deform_attn": types.ModuleType("rfdetr.models.ops.modules.ms_deform_attn"),
        "torch_linear_assignment": types.ModuleType("torch_linear_assignment"),
        "torch_linear_assignment.assignment": types.ModuleType("torch_linear_assignment.assignment"),
    }
    mods["rfdetr.models.matcher"].HungarianMatcher = HungarianMatcher
    mods["rfdetr.models.criterion"].SetCriterion = type(
        "SetCriterion", (), {"loss_boxes": lambda *a: "upstream", "loss_labels": lambda *a, **k: "upstream",
                             "focal_alpha": 0.25, "ia_bce_loss": True})
    mods["rfdetr.models.matcher"]._STACKED_COST_ELEMENT_LIMIT = 350_000
    msda = mods["rfdetr.models.ops.modules.ms_deform_attn"]
    msda.ms_deform_attn_core_pytorch = lambda *a, **k: "upstream"
    msda.MSDeformAttn = type("MSDeformAttn", (), {"forward": lambda self, *a, **k: "upstream", "_export": False})
    mods["rfdetr.models._assignment"]._assign_padded = lambda *a: "upstream"
    mods["torch_linear_assignment.assignment"].batch_linear_assignment = lambda c: "upstream"
    mods["torch_linear_assignment"].batch_linear_assignment = lambda c: "upstream"
    for name, mod in mods.items():
        monkeypatch.setitem(sys.modules, name, mod)
    return mods


def test_apply_patches_rebinds_the_reference_names(fake_rfdetr):
    done = patches.apply_patches("triton_matcher, cuda_lap,device_indices,stacked_costs,matcher,box_loss,label_loss")
    assert len(done) == 7 and all(":" in d for d in done)
    cls = fake_rfdetr["rfdetr.models.matcher"].HungarianMatcher
    assert fake_rfdetr["torch_linear_assignment.assignment"].batch_linear_assignment is matcher.batch_linear_assignment
    assert fake_rfdetr["torch_linear_assignment"].batch_linear_assignment is matcher.batch_linear_assignment
    assert fake_rfdetr["rfdetr.models.matcher"]._STACKED_COST_ELEMENT_LIMIT == 1 << 40
    assert cls.forward is matcher.HungarianMatcher.forward
    m = cls()
    # patched paths have no CPU fallback: host tensors raise instead of returning "upstream"
    outputs = {"pred_logits": torch.zeros(1, 3, 2), "pred_boxes": torch.zeros(1, 3, 4)}
    targets = [{"labels": torch.zeros(1, dtype=torch.int64), "boxes": torch.zeros(1, 4)}]
    with pytest.raises(ValueError, match="CUDA"):
        m._compute_compact_detection_cost_matrix(outputs, targets)
    with pytest.raises(ValueError, match="CUDA"):
        fake_rfdetr["rfdetr.models._assignment"]._assign_padded([torch.zeros(3, 1)], [1], 3, 1)
    crit = fake_rfdetr["rfdetr.models.criterion"].SetCriterion()
    with pytest.raises(ValueError, match="CUDA"):
        crit.loss_boxes({"pred_boxes": torch.zeros(1, 3, 4)}, targets,
                        [(torch.zeros(1, dtype=torch.int64), torch.zeros(1, dtype=torch.int64))], 1.0)
    with pytest.raises(ValueError, match="CUDA"):
        crit.loss_labels(outputs, targets, [(torch.zeros(1, dtype=torch.int64), torch.zeros(1, dtype=torch.int64))],
                         1.0)
    crit.use_varifocal_loss = True
    with pytest.raises(NotImplementedError):
        crit.loss_labels(outputs, targets, [(torch.zeros(1, dtype=torch.int64), torch.zeros(1, dtype=torch.int64))],
                         1.0)


def test_msda_patches_rebind_core_and_forward(fake_rfdetr):
    done = patches.apply_patches("fused_msda,fused_msda_native")
    assert len(done) == 2
    msda = fake_rfdetr["rfdetr.models.ops.modules.ms_deform_attn"]
    value = torch.zeros(1, 2, 4, 5)  # [B, M, D, S] on the host: the patched core has no CPU path
    locs6 = torch.zeros(1, 3, 2, 1, 2, 2)
    with pytest.raises(ValueError, match="CUDA"):
        msda.ms_deform_attn_core_pytorch(value, torch.tensor([[1, 5]]), locs6, torch.zeros(1, 3, 2, 1, 2))
    # the export layout (rank-5 locations) keeps the original core, export mode the original forward
    assert msda.ms_deform_attn_core_pytorch(value, None, torch.zeros(1, 3, 2, 2, 2), None) == "upstream"
    mod = msda.MSDeformAttn()
    mod._export = True
    assert mod.forward() == "upstream"


def test_unknown_patch_name_raises_keyerror():
    with pytest.raises(KeyError, match="unknown patch"):
        patches.apply_patches("not_a_patch")
    assert patches.apply_patches("") == []
