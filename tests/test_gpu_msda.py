"""rfm_msda_forward / _backward against a torch fp32 restatement of Deformable DETR's published core
(ms_deform_attn_core_pytorch: F.grid_sample per level, bilinear, align_corners=False, zero padding,
then the attention-weighted sum), on the reference's own verification cases (kernels_msda_cuda.py
CASES: the production decoder, encoder-sized queries, a single level) plus 64 channels per head (two
channel passes) and locations partly outside the map.  Tolerance: the reference's own bound,
2e-5 * max(1, scale) per output and per gradient (kernels_msda_cuda.py verify)."""

import pytest
import torch
import torch.nn.functional as F

from rfdetr_training_throughput_b200.msda import deformable_attention, module_forward

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda", 0)
TOL = 2e-5


def core_reference(value, shapes, locations, weights):
    """value [B, M, D, S] -> [B, Q, M * D], one grid_sample per level."""
    b, m, d, _s = value.shape
    _, q, _, levels, points, _ = locations.shape
    per_level = value.split([int(h) * int(w) for h, w in shapes.tolist()], dim=3)
    grids = 2 * locations - 1
    sampled = []
    for lid, (h, w) in enumerate(shapes.tolist()):
        v = per_level[lid].reshape(b * m, d, int(h), int(w))
        g = grids[:, :, :, lid].transpose(1, 2).flatten(0, 1)  # [B*M, Q, P, 2]
        sampled.append(F.grid_sample(v, g, mode="bilinear", padding_mode="zeros", align_corners=False))
    wts = weights.transpose(1, 2).reshape(b * m, 1, q, levels * points)
    out = (torch.stack(sampled, dim=-2).flatten(-2) * wts).sum(-1).view(b, m * d, q)
    return out.transpose(1, 2).contiguous()


def _case(batch, heads, head_dim, queries, points, shapes, spread=1.0, seed=7):
    g = torch.Generator(device="cuda").manual_seed(seed)
    seq = sum(h * w for h, w in shapes)
    value = torch.randn((batch, heads, head_dim, seq), device=DEV, generator=g)
    loc = (torch.rand((batch, queries, heads, len(shapes), points, 2), device=DEV, generator=g) - 0.5) * spread + 0.5
    w = torch.rand((batch, queries, heads, len(shapes), points), device=DEV, generator=g)
    w = w / w.sum(-1, keepdim=True)
    return value, torch.tensor(shapes, device=DEV, dtype=torch.int64), loc, w


CASES = [
    ("production decoder", dict(batch=8, heads=8, head_dim=32, queries=300, points=4, shapes=[(36, 36), (18, 18), (9, 9)])),
    ("encoder-sized queries", dict(batch=4, heads=8, head_dim=32, queries=1296, points=4, shapes=[(36, 36), (18, 18)])),
    ("single level", dict(batch=2, heads=4, head_dim=16, queries=64, points=4, shapes=[(20, 20)])),
    ("64 channels", dict(batch=2, heads=4, head_dim=64, queries=100, points=2, shapes=[(12, 17), (6, 9)])),
    ("outside the map", dict(batch=2, heads=8, head_dim=32, queries=200, points=4, shapes=[(16, 16), (8, 8)],
                             spread=1.6)),
]


@pytest.mark.parametrize("name,case", CASES, ids=[c[0] for c in CASES])
def test_msda_matches_grid_sample_core(name, case):
    value, shapes, loc, w = _case(**case)
    ours_in = [t.clone().requires_grad_(True) for t in (value, loc, w)]
    ref_in = [t.clone().requires_grad_(True) for t in (value, loc, w)]
    out = deformable_attention(ours_in[0], shapes, ours_in[1], ours_in[2])
    ref = core_reference(ref_in[0], shapes, ref_in[1], ref_in[2])
    seed = torch.randn(ref.shape, device=DEV, generator=torch.Generator(device="cuda").manual_seed(3))
    out.backward(seed)
    ref.backward(seed)
    torch.cuda.synchronize()
    pairs = {"output": (out, ref), "grad_value": (ours_in[0].grad, ref_in[0].grad),
             "grad_locations": (ours_in[1].grad, ref_in[1].grad), "grad_weights": (ours_in[2].grad, ref_in[2].grad)}
    for what, (a, b) in pairs.items():
        scale = max(1.0, float(b.abs().max()))
        assert float((a - b).abs().max()) <= TOL * scale, what


class _Module(torch.nn.Module):
    """The projections of an MSDeformAttn module (d_model 256, 8 heads, 3 levels, 4 points)."""

    def __init__(self, d_model=256, heads=8, levels=3, points=4):
        super().__init__()
        self.d_model, self.n_heads, self.n_levels, self.n_points = d_model, heads, levels, points
        self.sampling_offsets = torch.nn.Linear(d_model, heads * levels * points * 2)
        self.attention_weights = torch.nn.Linear(d_model, heads * levels * points)
        self.value_proj = torch.nn.Linear(d_model, d_model)
        self.output_proj = torch.nn.Linear(d_model, d_model)


def test_module_forward_matches_the_unfused_module():
    torch.manual_seed(0)
    mod = _Module().to(DEV)
    shapes = torch.tensor([(36, 36), (18, 18), (9, 9)], device=DEV, dtype=torch.int64)
    start = torch.tensor([0, 1296, 1620], device=DEV, dtype=torch.int64)
    query = torch.randn(2, 300, 256, device=DEV)
    ref_pts = torch.rand(2, 300, 3, 4, device=DEV) * 0.5 + 0.25  # cxcywh reference boxes
    flat = torch.randn(2, 1701, 256, device=DEV)
    out = module_forward(mod, query, ref_pts, flat, shapes, start)
    # the same module written with the grid_sample core
    value = mod.value_proj(flat).view(2, 1701, 8, 32)
    offsets = mod.sampling_offsets(query).view(2, 300, 8, 3, 4, 2)
    w = F.softmax(mod.attention_weights(query).view(2, 300, 8, 12), -1).view(2, 300, 8, 3, 4)
    loc = ref_pts[:, :, None, :, None, :2] + offsets / 4 * ref_pts[:, :, None, :, None, 2:] * 0.5
    ref = mod.output_proj(core_reference(value.permute(0, 2, 3, 1), shapes, loc, w))
    torch.cuda.synchronize()
    assert float((out - ref).abs().max()) <= TOL * max(1.0, float(ref.abs().max()))
