"""The CUDA annotation rasteriser paints exactly the CPU oracle's pixels."""
import numpy as np
import pytest
import torch

from predicitivecoding_b200 import ops
from predicitivecoding_b200.systems import imaging as im
from predicitivecoding_b200.systems import vision as vi

pytestmark = pytest.mark.gpu


def test_annotation_kernel_matches_cpu():
    rng = np.random.default_rng(3)
    base = rng.integers(0, 256, (120, 160, 3), dtype=np.uint8)
    tracks = []
    for i in range(12):
        t = vi.Track(i + 1, vi.Detection(*sorted(rng.uniform(-20, 180, 2)), *sorted(rng.uniform(-20, 140, 2))))
        t.cx, t.cy = rng.uniform(0, 160), rng.uniform(0, 120)
        tracks.append(t)
    ann = (vi.Annotator(3).draw_boxes([vi.Detection(10, 10, 60, 90)]).draw_tracks(tracks)
           .draw_line(-10, 5, 170, 115).draw_line(80, 0, 80, 119, thickness=4)
           .draw_zone([(20, 20), (140, 30), (100, 110), (15, 100)]))
    cpu = ann.render_cpu(im.RgbImage.from_pixel_data(base, 160, 120)).pixels
    gpu = torch.from_numpy(base.copy()).cuda()
    before = ops.launch_count()
    ann.render_cuda(gpu)
    torch.cuda.synchronize()
    assert ops.launch_count() == before + 3
    assert np.array_equal(gpu.cpu().numpy(), cpu)
