"""ONNX export of the plugin node, traced on the CPU.

The reference exports its CUDA path as one custom_ops::LocalCorrCudaPyramid
node (blocks.py:156-204 for the RAFT block, blocks.py:951-1043 for the
single-level spatial form) that its TensorRT plugin computes. Serialising a
model needs the `onnx` package, which is not installed here, so these tests
stop one step earlier: they build the exporter's ONNX graph (TorchScript
exporter, opset 17) with the export flag set and check the node, its
attributes and its output shape.
"""

import math

import pytest
import torch

import localcorr_b200 as lc

try:
    from torch.onnx._internal.torchscript_exporter import _globals as _G
    from torch.onnx._internal.torchscript_exporter import utils as _U
except ImportError:  # pragma: no cover - torch without the TorchScript exporter
    _G = _U = None

pytestmark = pytest.mark.skipif(_U is None, reason="TorchScript ONNX exporter not available")


def _onnx_graph(model, args):
    _G.GLOBALS.export_onnx_opset_version = 17
    _G.GLOBALS.in_onnx_export = True
    try:
        with _U.exporter_context(model, torch.onnx.TrainingMode.EVAL, False):
            graph, _, _ = _U._model_to_graph(
                model, args, operator_export_type=torch.onnx.OperatorExportTypes.ONNX)
    finally:
        _G.GLOBALS.in_onnx_export = False
    return graph


def _plugin_nodes(graph):
    return [n for n in graph.nodes() if n.kind() == "custom_ops::LocalCorrCudaPyramid"]


class _Raft(torch.nn.Module):
    def forward(self, f1, f2, coords):
        block = lc.get_localcorr_block(f1, f2, num_levels=3, radius=4, corr_mode="localcorr_cuda")
        return block(coords)


class _Pwc(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.sampler = lc.get_localcorr_sampler(patch_size=7, corr_mode="localcorr_cuda")

    def forward(self, a, b):
        return self.sampler(a, b)


def test_block_exports_one_plugin_node():
    b, c, h, w = 2, 16, 24, 32
    args = (torch.randn(b, c, h, w), torch.randn(b, c, h, w), torch.randn(b, 2, h, w))
    graph = _onnx_graph(_Raft(), args)
    nodes = _plugin_nodes(graph)
    assert len(nodes) == 1
    n = nodes[0]
    assert n.i("radius") == 4 and n.i("levels") == 3 and n.i("dilation") == 1
    assert n.i("ymajor") == 0
    assert n.output().type().sizes() == [b, 3, 81, h, w]
    # inputs: NHWC fmap1, the batch-major packed pyramid, the coords
    ins = list(n.inputs())
    assert ins[0].type().sizes() == [b, h, w, c]
    packed = sum(c * (h >> l) * (w >> l) for l in range(3))
    assert ins[1].type().sizes() == [b, packed]
    assert ins[2].type().sizes() == [b, 2, h, w]
    kinds = [x.kind() for x in graph.nodes()]
    assert "onnx::Div" in kinds  # the block's 1/sqrt(C) outside the plugin
    outs = list(graph.outputs())
    assert outs[0].type().sizes() == [b, 3 * 81, h, w]


def test_sampler_exports_single_level_ymajor_node():
    b, c, h, w = 1, 8, 12, 20
    graph = _onnx_graph(_Pwc(), (torch.randn(b, c, h, w), torch.randn(b, c, h, w)))
    nodes = _plugin_nodes(graph)
    assert len(nodes) == 1
    n = nodes[0]
    assert n.i("radius") == 3 and n.i("levels") == 1 and n.i("ymajor") == 1
    assert n.i("dilation") == 1
    # the node's [B, 1, 49, H, W] is reshaped to the sampler's [B, 7, 7, H, W]
    (reshape,) = [u.user for u in n.output().uses() if u.user.kind() == "onnx::Reshape"]
    shape = reshape.inputsAt(1).node()
    assert shape.kind() == "onnx::Constant"
    assert shape.t("value").tolist() == [b, 7, 7, h, w]


def test_spatial_block_export_keeps_dilation_and_scale():
    b, c, h, w = 1, 9, 10, 14
    f1, f2 = torch.randn(b, c, h, w), torch.randn(b, c, h, w)

    class _Fnc(torch.nn.Module):
        def forward(self, x, y):
            blk = lc.LocalCorrCudaPyramidSpatialBlock(x, y, radius=2, dilation=2,
                                                      normalize="sqrt")
            return blk()

    graph = _onnx_graph(_Fnc(), (f1, f2))
    (n,) = _plugin_nodes(graph)
    assert n.i("radius") == 2 and n.i("dilation") == 2 and n.i("levels") == 1
    muls = [x for x in graph.nodes() if x.kind() == "onnx::Mul"]
    assert muls, "normalize='sqrt' scales the plugin output"
    consts = [x.t("value").item() for x in graph.nodes()
              if x.kind() == "onnx::Constant" and x.t("value").numel() == 1]
    assert any(abs(v - 1.0 / math.sqrt(c)) < 1e-6 for v in consts)
