"""Host-side structure of the DPT head (model.Decoder) without a GPU: the
launch count the bench reports for the depth model."""
import torch

from beatlm_b200 import model


def test_head_launch_count_follows_its_structure():
    """DPT-S (neck 48/96/192/384): projections and necks 16, the transposed
    convolutions 2 (48 channels, from the projection's rows) and 3 (96), the
    strided one 2; fusion 6 + 3 x 10; head 6: 65 launches."""
    dc = model.DecoderConfig()
    d = model.Decoder.__new__(model.Decoder)
    d.dcfg = dc
    d.stages = [{"c": c, "resample": rs, "proj": (torch.empty((-(-c // 32) * 32, 64)),)}
                for c, rs in zip(dc.neck, dc.reassemble)]
    d.fusion = [None] * len(dc.neck)
    assert d.launches_per_frame() == 65
