"""Device pre/post-processing against the torch restatement of the policy's processing."""

import pytest
import torch

from oracle import processing as P

DEV = "cuda"


@pytest.mark.gpu
@pytest.mark.parametrize("n,c,h,w", [(2, 3, 256, 256), (1, 3, 480, 640), (3, 3, 512, 512), (1, 3, 300, 200)])
def test_prepare_images_matches_interpolate_and_pad(n, c, h, w):
    from smolvla_mujoco_libero_b200 import processing
    g = torch.Generator().manual_seed(h * 7 + w)
    x = torch.rand(n, c, h, w, generator=g)
    got = processing.prepare_images(x.to(DEV)).cpu()
    ref = P.prepare_images(x)
    assert got.shape == ref.shape == (n, c, 512, 512)
    # source indices are fp32: near 512 their spacing is 2^-14, so an index may round one ulp differently from
    # torch's, moving a bilinear weight by up to 2^-14 (times a neighbour difference <= 1, doubled by x*2-1)
    assert float((got - ref).abs().max()) <= 2 * 2.0 ** -14


@pytest.mark.gpu
def test_prepare_images_from_camera_frames_into_a_strided_buffer():
    from smolvla_mujoco_libero_b200 import processing
    g = torch.Generator().manual_seed(5)
    frames = torch.randint(0, 256, (2, 256, 256, 3), generator=g, dtype=torch.uint8)
    buf = torch.zeros(2, 2, 3, 512, 512, device=DEV)  # [B, cams, C, H, W]: camera 1 of every sample
    processing.prepare_images(frames.to(DEV), out=buf[:, 1])
    ref = P.prepare_images(frames)
    assert float((buf[:, 1].cpu() - ref).abs().max()) <= 2e-6
    assert int(buf[:, 0].count_nonzero()) == 0


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["mean_std", "min_max"])
def test_state_and_action_normalisation(mode):
    from smolvla_mujoco_libero_b200 import processing
    g = torch.Generator().manual_seed(11)
    if mode == "mean_std":
        st = {"mean": torch.randn(8, generator=g), "std": torch.rand(8, generator=g) + 0.1}
        at = {"mean": torch.randn(7, generator=g), "std": torch.rand(7, generator=g) + 0.1}
    else:
        st = {"min": -torch.rand(8, generator=g) - 0.5, "max": torch.rand(8, generator=g) + 0.5}
        at = {"min": -torch.rand(7, generator=g) - 0.5, "max": torch.rand(7, generator=g) + 0.5}
    state = torch.randn(4, 8, generator=g)
    acts = torch.randn(4, 50, 32, generator=g)
    dev = lambda d: {k: v.to(DEV) for k, v in d.items()}  # noqa: E731
    s = processing.prepare_state(state.to(DEV), dev(st), 32).cpu()
    a = processing.unnormalize_actions(acts.to(DEV), dev(at), 7).cpu()
    assert torch.allclose(s, P.prepare_state(state, st, 32), rtol=0, atol=1e-6)
    assert torch.allclose(a, P.unnormalize_actions(acts, at, 7), rtol=0, atol=1e-6)
