"""The model shape tables (3x3 convs of alexnet / resnet18 / resnet34 / vgg16 at 224x224)
against torchvision's own modules, as the reference extracts them with forward hooks
(benchmarks/e2e_benchmark.py:91-137)."""
import pytest

import model_shapes


def _hooked(name):
    torch = pytest.importorskip("torch")
    models = pytest.importorskip("torchvision.models")
    m = getattr(models, name)(weights=None).eval()
    out = []

    def hook(mod, inp, _):
        out.append(model_shapes.ConvShape(mod.in_channels, mod.out_channels, inp[0].shape[2],
                                          inp[0].shape[3], mod.stride[0], mod.padding[0]))

    hs = [mod.register_forward_hook(hook) for mod in m.modules()
          if isinstance(mod, torch.nn.Conv2d) and mod.kernel_size == (3, 3)]
    with torch.no_grad():
        m(torch.zeros(1, 3, 224, 224))
    for h in hs:
        h.remove()
    return out


@pytest.mark.parametrize("name", sorted(model_shapes.MODELS))
def test_tables_match_torchvision(name):
    assert model_shapes.conv3x3_layers(name) == _hooked(name)


def test_stride1_counts_and_chaining():
    assert [len(model_shapes.stride1_layers(m))
            for m in ("alexnet", "resnet18", "resnet34", "vgg16")] == [3, 13, 29, 13]
    layers = model_shapes.stride1_layers("vgg16")
    assert all(model_shapes.chains(a, b) == ((a.h, a.c_out) == (b.h, b.c_in))
               for a, b in zip(layers, layers[1:]))
    assert not model_shapes.chains(None, layers[0])
