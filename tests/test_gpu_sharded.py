"""ShardedEngine on one GPU: the split by image (uneven shards included), the per-device threads and the
concatenation in image order must reproduce one engine's output bit for bit, since every image's logits
are independent of its batch mates."""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(("devices", "B"), [([0, 0], 5), ([0, 0, 0], 7), ([0, 0, 0], 2)])
def test_sharded_engine_matches_one_engine(cuda_device, no_device_error, devices, B):
    from foidfinder_b200.config import EVA02_L
    from foidfinder_b200.engine import Engine
    from foidfinder_b200.multigpu import ShardedEngine, shard_sizes

    cfg = EVA02_L.with_(name="sharded-112", image_size=112, depth=2)
    imgs = torch.randint(0, 256, (B, 112, 112, 3), generator=torch.Generator().manual_seed(21), dtype=torch.uint8)
    one = Engine(cfg, device=0, seed=7)
    ref_logits, ref_idx, ref_val = (t.cpu() for t in one.forward(imgs))
    torch.cuda.synchronize()
    one.close()
    sharded = ShardedEngine(cfg, devices, seed=7)
    try:
        assert sorted(shard_sizes(B, len(devices))) != [B // len(devices)] * len(devices) or B % len(devices) == 0
        logits, idx, val = sharded.forward(imgs)
        assert logits.device.type == "cpu" and logits.shape == (B, cfg.num_tags)
        assert torch.equal(logits, ref_logits)
        assert torch.equal(idx, ref_idx) and torch.equal(val, ref_val)
        l2, i2, v2 = sharded.forward(imgs, topk=False)
        assert i2 is None and v2 is None and torch.equal(l2, ref_logits)
    finally:
        sharded.close()
