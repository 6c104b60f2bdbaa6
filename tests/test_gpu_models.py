"""Model shape feed on the GPU: every stride-1 3x3 conv of resnet18, resnet34 and vgg16 (at a
224x224 input) runs as a chained stack through cwg_conv3x3_fused; each layer's output for
image 0 is checked against the reference C on the exact input that layer received."""
import pytest

import model_shapes
from conftest import assert_close
from test_gpu_parity import oracle_conv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(model_shapes.MODELS))
def test_model_stack_matches_reference(cuda_dev, name):
    layers = model_shapes.stride1_layers(name)
    times, kept, prepared = model_shapes.run_stack(name, 2, cuda_dev, 0,
                                                   keep=set(range(len(layers))))
    assert len(times) == len(layers) and all(t > 0 for t in times)
    assert len(kept) == len(layers)
    for (i, s, x, y), (_, _, _, g, bias) in zip(kept, prepared):
        xs = x[:1].float().cpu().numpy()
        ys = y[:1].float().cpu().numpy()
        assert_close(ys, oracle_conv(xs, g, bias, 2, True), "f23", f"{name} layer {i} {s}")


def test_model_stack_graph_replay_matches_eager(cuda_dev):
    """The stack captured into one CUDA graph (launches only, no host work per layer)
    reproduces the eager stack's final output."""
    import torch

    import cwg

    name = "resnet18"
    replay, y_graph = model_shapes.capture_stack(name, 1, cuda_dev, cwg.NO_SPLIT)
    replay()
    torch.cuda.synchronize()
    n_layers = len(model_shapes.stride1_layers(name))
    _, kept, _ = model_shapes.run_stack(name, 1, cuda_dev, cwg.NO_SPLIT, keep={n_layers - 1})
    torch.testing.assert_close(y_graph, kept[0][3], rtol=0, atol=0)
