"""Multimodal datasets: OBELICS (parquet / JSONL) and CC12M (WebDataset tar) readers, the
native-resolution image pipeline, packing, collation and the Qwen3-VL model on the batches."""
import io
import json
import os
import tarfile

import pytest
import torch

from torchtitan_b200.components.loss import IGNORE_INDEX
from torchtitan_b200.components.mm_datasets import (MMDataLoader, MultiModalCollator, SamplePacker, VisionSpec,
                                                     build_sample, read_cc12m, smart_resize, vision_to_patches)
from torchtitan_b200.components.tokenizer import SyntheticTokenizer

SPECIAL = dict(image_token_id=2046, video_token_id=2047, vision_start_id=2040, vision_end_id=2041)


def _png(h, w, seed):
    from PIL import Image

    g = torch.Generator().manual_seed(seed)
    arr = torch.randint(0, 256, (h, w, 3), generator=g, dtype=torch.uint8).numpy()
    buf = io.BytesIO()
    Image.fromarray(arr).save(buf, format="PNG")
    return buf.getvalue()


def _cc12m_shards(d, n=6):
    os.makedirs(d, exist_ok=True)
    for shard in range(2):
        with tarfile.open(os.path.join(d, f"shard-{shard:05d}.tar"), "w") as tar:
            for i in range(n // 2):
                key = f"{shard:02d}{i:04d}"
                for ext, data in (("png", _png(40 + 8 * i, 70, shard * 10 + i)),
                                  ("txt", f"caption {shard} {i}".encode()), ("json", b"{}")):
                    info = tarfile.TarInfo(f"{key}.{ext}")
                    info.size = len(data)
                    tar.addfile(info, io.BytesIO(data))


def test_smart_resize_rule():
    assert smart_resize(100, 200, 32, 65536, 16777216) == (192, 384)  # grown to the minimum area
    h, w = smart_resize(3000, 4000, 32, 65536, 1 << 20)  # shrunk under the maximum area
    assert h % 32 == 0 and w % 32 == 0 and h * w <= 1 << 20 and abs(w / h - 4 / 3) < 0.05
    assert smart_resize(256, 512, 32, 1024, 1 << 24) == (256, 512)
    with pytest.raises(ValueError):
        smart_resize(10, 3000, 32, 1024, 1 << 24)


def test_patches_match_the_model_layout():
    """An image's patch rows equal the layout the Qwen3-VL tower was tested with (the image
    repeated over the temporal patch, merge groups consecutive)."""
    from torchtitan_b200.components.mm_dataloader import patchify

    spec = VisionSpec(patch_size=8, temporal_patch_size=2, merge_size=2)
    img = torch.randn(3, 32, 48)
    a, ga = vision_to_patches(img.permute(1, 2, 0)[None], spec)
    b, gb = patchify(img, 8, 2, 2)
    assert ga == gb == [1, 4, 6] and torch.equal(a, b)
    # a 3-frame clip pads to 4 frames with its last frame: two temporal patches
    clip = torch.randn(3, 32, 48, 3)
    p, g = vision_to_patches(clip, spec)
    assert g == [2, 4, 6] and p.shape == (48, 3 * 2 * 64)
    q, _ = vision_to_patches(torch.cat([clip, clip[-1:]]), spec)
    assert torch.equal(p, q)


def test_cc12m_loader_batches(tmp_path):
    _cc12m_shards(str(tmp_path))
    recs = list(read_cc12m(str(tmp_path)))
    assert len(recs) == 6 and recs[0]["texts"][1] == "caption 0 0"
    tok = SyntheticTokenizer(SyntheticTokenizer.Config(vocab_size=2048))
    cfg = MMDataLoader.Config(dataset="cc12m", dataset_path=str(tmp_path), infinite=False, patch_size=8,
                              min_pixels=32 * 32, max_pixels=64 * 64, **SPECIAL)
    dl = MMDataLoader(cfg, tokenizer=tok, seq_len=96, local_batch_size=2)
    batches = list(dl)
    assert len(batches) == 3
    inp, labels = batches[0]
    assert inp["input"].shape == (2, 96) and labels.shape == (2, 96)
    n_img = int((inp["input"] == 2046).sum())
    grid = inp["grid_thw"]
    assert grid.shape == (2, 3) and n_img == int((grid.prod(1) // 4).sum())
    assert inp["pixel_values"].shape == (int(grid.prod(1).sum()), 3 * 2 * 64)
    # placeholders and vision brackets never count toward the loss
    assert not (labels == 2046).any() and not (labels == 2040).any() and not (labels == 2041).any()
    # two dp ranks split the records
    got = [sum(1 for _ in MMDataLoader(cfg, tokenizer=tok, seq_len=96, local_batch_size=1, dp_world_size=2,
                                       dp_rank=r)) for r in range(2)]
    assert got == [3, 3]


def test_obelics_interleaved_parquet_and_jsonl(tmp_path):
    import base64

    import pyarrow as pa
    import pyarrow.parquet as pq

    rows = {"texts": [["intro", None, "middle", None, "end"], [None, "only caption"]],
            "images": [[None, _png(64, 64, 1), None, _png(32, 96, 2), None], [_png(50, 50, 3), None]]}
    pq.write_table(pa.table(rows), str(tmp_path / "a.parquet"))
    with open(tmp_path / "b.jsonl", "w") as f:
        f.write(json.dumps({"texts": ["hi", None], "images": [None, {"bytes": base64.b64encode(
            _png(40, 40, 4)).decode()}]}) + "\n")
    tok = SyntheticTokenizer(SyntheticTokenizer.Config(vocab_size=2048))
    spec = VisionSpec(patch_size=8, min_pixels=16 * 16, max_pixels=64 * 64)
    from torchtitan_b200.components.mm_datasets import read_obelics

    recs = list(read_obelics(str(tmp_path)))
    assert len(recs) == 3
    ids = {"image": 2046, "video": 2047, "vision_start": 2040, "vision_end": 2041}
    s = build_sample(recs[0], tok, spec, ids)
    assert len(s["pixel_values"]) == 2
    t = s["input_ids"].tolist()
    # text, [start, pads, end], text, [start, pads, end], text, eos
    starts = [i for i, v in enumerate(t) if v == 2040]
    assert len(starts) == 2 and t[:5] == tok.encode("intro") and t[-1] == tok.eos_id
    n0 = t.index(2041) - starts[0] - 1
    assert n0 == (s["pixel_values"][0].shape[1] // 16) * (s["pixel_values"][0].shape[2] // 16)
    assert (s["labels"] == IGNORE_INDEX).sum() == sum(1 for v in t if v in (2040, 2041, 2046))
    assert build_sample({"texts": ["a", None], "images": [None, b"not an image"]}, tok, spec, ids) is None


def test_packing_and_resume(tmp_path):
    _cc12m_shards(str(tmp_path), n=8)
    tok = SyntheticTokenizer(SyntheticTokenizer.Config(vocab_size=2048))
    cfg = MMDataLoader.Config(dataset="cc12m", dataset_path=str(tmp_path), infinite=True, patch_size=8,
                              min_pixels=32 * 32, max_pixels=48 * 48, packing_buffer_size=4, **SPECIAL)
    dl = MMDataLoader(cfg, tokenizer=tok, seq_len=128, local_batch_size=2)
    it = iter(dl)
    first = [next(it) for _ in range(3)]
    # packed rows hold several samples: positions restart inside a row
    pos = first[0][0]["positions"]
    assert int((pos[:, 1:] == 0).logical_and(first[0][0]["input"][:, 1:] != 0).sum()) > 0
    st = dl.state_dict()
    want = [next(it) for _ in range(2)]
    dl2 = MMDataLoader(cfg, tokenizer=tok, seq_len=128, local_batch_size=2)
    dl2.load_state_dict(st)
    it2 = iter(dl2)
    got = [next(it2) for _ in range(2)]
    for (a, la), (b, lb) in zip(want, got):
        assert torch.equal(a["input"], b["input"]) and torch.equal(la, lb)


def test_packer_scan_and_pick():
    mk = lambda n: {"input_ids": torch.full((n,), n), "labels": torch.full((n,), n),  # noqa: E731
                    "positions": torch.arange(n), "pixel_values": [], "pixel_values_videos": []}
    p = SamplePacker(10, buffer_size=4)
    for n in (6, 5, 4, 3):
        p.add(mk(n))
    a = p.pop()  # 6 + 4 fill a sequence (5 does not fit after 6; the scan goes on)
    assert a["input_ids"].tolist() == [6] * 6 + [4] * 4
    assert p.pop() is None  # 5 + 3 is not full: it waits for more samples
    p.add(mk(2))
    assert p.pop() is None  # the buffer (5, 3, 2) is below its size: no packing yet
    p.add(mk(1))
    assert p.pop()["input_ids"].tolist() == [5] * 5 + [3] * 3 + [2] * 2
    p.add(mk(11))
    p.flush()
    assert p.pop()["input_ids"].tolist() == [1]  # the flush emits the leftover
    assert p.pop() is None  # and the sample longer than a sequence was dropped


def test_collator_caps_images_per_batch():
    spec = VisionSpec(patch_size=8)
    mk = lambda k: {"input_ids": torch.arange(5), "labels": torch.arange(5), "positions": torch.arange(5),  # noqa
                    "pixel_values": [torch.randn(1, 16, 16, 3)] * k, "pixel_values_videos": []}
    out, lab = MultiModalCollator(3, 8, spec, max_images_per_batch=3)([mk(2), mk(1), mk(2)])
    assert out["grid_thw"].shape[0] == 3 and out["input"].shape == (3, 8)
    assert (out["input"][2] == 0).all() and (lab[2] == IGNORE_INDEX).all()  # the dropped sample is padding


def test_qwen3_vl_trains_on_cc12m_batches(tmp_path):
    from torchtitan_b200.components.loss import cross_entropy_loss
    from torchtitan_b200.models.qwen3_vl import model_registry

    _cc12m_shards(str(tmp_path))
    spec = model_registry("debugmodel")
    torch.manual_seed(0)
    m = spec.model.build()
    m.init_weights()
    a = m.model_args
    va = m.vision_encoder
    tok = SyntheticTokenizer(SyntheticTokenizer.Config(vocab_size=2048))
    P = va.patch_size if hasattr(va, "patch_size") else 16
    cfg = MMDataLoader.Config(dataset="cc12m", dataset_path=str(tmp_path), infinite=False, patch_size=P,
                              spatial_merge_size=a.spatial_merge_size, min_pixels=(2 * P) ** 2,
                              max_pixels=(4 * P) ** 2, **SPECIAL)
    inp, labels = next(iter(MMDataLoader(cfg, tokenizer=tok, seq_len=64, local_batch_size=2)))
    kw = {k: v for k, v in inp.items() if k not in ("input", "special_tokens")}
    logits = m(inp["input"], **kw)
    loss = cross_entropy_loss(logits, labels) / (labels != IGNORE_INDEX).sum()
    loss.backward()
    assert torch.isfinite(loss) and m.vision_encoder.patch_embed.weight.grad.abs().sum() > 0


def test_trainer_steps_on_cc12m_config(tmp_path):
    from torchtitan_b200.config.manager import ConfigManager
    from torchtitan_b200.trainer import Trainer

    _cc12m_shards(str(tmp_path / "data"))
    t = Trainer(ConfigManager().parse_args([
        "--module", "qwen3_vl", "--config", "qwen3_vl_debugmodel_cc12m", "--dataloader.dataset-path",
        str(tmp_path / "data"), "--training.seq-len", "256", "--training.steps", "2", "--training.dtype",
        "float32", "--training.mixed-precision-param", "float32", "--dump-folder", str(tmp_path / "out")]))
    it = t.batch_generator(t.dataloader)
    for _ in range(2):
        t.step += 1
        assert torch.isfinite(t.train_step(it))
    t.close()
