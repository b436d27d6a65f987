"""Host logic: LayerInputs.packed lays a whole step's inputs out as views of
one flat buffer (one host->device copy per step)."""
import torch

from dsv4attn.layer import LayerInputs
from dsv4attn.tables import PathArgs


def test_packed_views_cover_one_buffer_without_overlap():
    a = PathArgs()
    flat, layers = LayerInputs.packed(a, 4, 3, device="cpu")
    assert len(layers) == 3
    spans = []
    base = flat.data_ptr()
    for L, ref in zip(layers, [LayerInputs.empty(a, 4, "cpu")] * 3):
        for t, r in zip(L.tensors(), ref.tensors()):
            assert t.shape == r.shape and t.dtype == r.dtype and t.is_contiguous()
            off = t.data_ptr() - base
            assert off % 256 == 0
            spans.append((off, off + t.numel() * t.element_size()))
    spans.sort()
    assert spans[-1][1] <= flat.numel()
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 <= b0
    # writes through a view land in the flat buffer
    layers[1].iw.fill_(2.5)
    off = layers[1].iw.data_ptr() - base
    assert torch.equal(flat[off:off + 4].view(torch.float32), torch.tensor([2.5]))
