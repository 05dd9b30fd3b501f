"""Data pipeline on CPU: sample-data formats, budget packing, exact resume, batch assembly."""
import itertools
import math

import pytest
import torch

from pan2_b200.data.items import Budgets, HashCaptionCodec
from pan2_b200.data.loader import PackedLoader
from pan2_b200.data.make_sample_data import write_sample_data
from pan2_b200.data.packing import CsvStream, DataloaderState, PackingDataset, read_csv_row

from tiny import tiny_model


@pytest.fixture(scope="module")
def sample_dir(tmp_path_factory):
    d = tmp_path_factory.mktemp("sample")
    write_sample_data(str(d), num_videos=7, num_images=6, latent_frames=3, height=8, width=12, channels=48,
                      image_grids=((8, 8), (6, 10), (4, 4)))
    return d


def _dataset(d, resume=None, image_prob=0.4, **over):
    budgets = Budgets(joint=400, video=360, caption=160, text_encoder=220, joint_segment=400, caption_segment=80,
                      max_num_seq=4)
    kw = dict(patch_size=(1, 2, 2), rope_axes=(8, 12, 12), num_buffers=2, seed=3, image_tars=[str(d / "images.tar")],
              image_sample_prob=image_prob, image_cond_prob=0.5, cfg_drop_prob=0.2, num_workers=2, resume=resume,
              pad_multiple=16)
    kw.update(over)
    return PackingDataset([str(d / "videos.csv")], HashCaptionCodec(embed_dim=64), budgets, **kw)


def _sig(plan):
    return [(it.modality, it.ref.global_index, it.ref.shard_index, it.ref.sample_index, it.ref.epoch_index,
             it.ref.cycle, it.prefix_frames, it.caption.cropped_length) for it in plan.items]


def test_csv_rows_and_offsets(sample_dir):
    s = CsvStream([str(sample_dir / "videos.csv")])
    rows = list(itertools.islice(s.rows(None), 9))
    assert [r.global_index for _, r in rows] == list(range(9))
    assert rows[7][1].epoch_index == 1 and rows[7][1].local_index == 0
    assert "\n" in rows[2][0]["caption"]  # multi-line quoted field
    for row, ref in rows[:7]:
        assert read_csv_row(str(sample_dir / "videos.csv"), ref.local_file_pos) == row
    # resume after row 4 continues at row 5
    nxt = next(s.rows(rows[4][1]))
    assert nxt[1].global_index == 5 and nxt[0] == rows[5][0]


def test_packing_budgets(sample_dir):
    ds = _dataset(sample_dir)
    plans = list(itertools.islice(iter(ds), 8))
    b = ds.budgets
    seen = set()
    for p in plans:
        assert sum(p.video_lens) <= b.video
        assert sum(p.video_lens) + sum(p.caption_lens) <= b.joint
        assert sum(p.caption_lens) <= b.caption
        assert sum(it.caption.full_length for it in p.items) <= b.text_encoder
        assert len(p.items) <= b.max_num_seq
        assert p.total % 16 == 0 and p.total >= sum(p.video_lens) + sum(p.caption_lens)
        assert p.freqs_cos.shape == (p.total, 32)
        for it in p.items:
            key = (it.modality, it.ref.global_index, it.ref.shard_index, it.ref.sample_index, it.ref.cycle)
            assert key not in seen
            seen.add(key)
    mods = {it.modality for p in plans for it in p.items}
    assert mods == {"video", "image"}


def test_resume_is_exact(sample_dir):
    full = list(itertools.islice(iter(_dataset(sample_dir)), 10))
    for k in (2, 5):
        st = DataloaderState.from_json(full[k].state.to_json())
        resumed = list(itertools.islice(iter(_dataset(sample_dir, resume=st)), 10 - k - 1))
        assert [_sig(p) for p in resumed] == [_sig(p) for p in full[k + 1:]]


def test_reset_video_stream(sample_dir):
    full = list(itertools.islice(iter(_dataset(sample_dir)), 4))
    st = full[2].state.reset_video_stream()
    assert st.next_stream_ref is None
    assert all(r.modality == "image" for b in st.buffer_items for r in b)
    plans = list(itertools.islice(iter(_dataset(sample_dir, resume=st)), 2))
    assert plans


def test_loader_assembly_feeds_model(sample_dir):
    ds = _dataset(sample_dir, image_prob=0.0)
    loader = PackedLoader(ds, device="cpu", dtype=torch.float32, seed=0, shift=3.0)
    batch, meta = next(iter(loader))
    loader.close()
    P = batch["packed_seq_params"]
    assert batch["hidden_states"].shape == (97 * 4, P.n_video, 1, 1)
    assert batch["target"].shape == (P.n_video, 48 * 4)
    assert batch["text_states"].shape == (P.n_text, 64)
    assert meta.active_joint_length == P.n_active
    assert meta.dataloader_state is not None
    # mask channel is 1 exactly on conditioned frames
    tok = 0
    hs = batch["hidden_states"][:, :, 0, 0]
    for vl, nt in zip(P.video_lens, P.caption_lens):
        assert set(hs[96 * 4:97 * 4, tok:tok + vl].unique().tolist()) <= {0.0, 1.0}
        tok += vl
    model = tiny_model(text_embed_dim=64, hidden_size=128, rope_axes_dim=(8, 12, 12))
    loss = model(**batch)
    assert torch.isfinite(loss) and loss.item() > 0


def test_synthetic_workload_batches_fit_their_budgets():
    from pan2_b200.data.cp_batch import strided_split
    from pan2_b200.data.synthetic import sft_mix_items, synthetic_items_batch, synthetic_packed_batch
    items = sft_mix_items(109142, 110576, 8, 512, seed=3)
    n_video = sum(t * (h // 2) * (w // 2) for (t, h, w), _ in items)
    assert len(items) <= 8 and n_video <= 109142 and n_video + 512 * len(items) <= 110576
    assert sum(1 for (t, _, _), _ in items if t == 1) == 4  # single-frame image items
    small = [((3, 8, 8), True), ((1, 8, 8), False), ((5, 8, 8), False)]
    b = synthetic_items_batch(small, [16, 8, 12], text_dim=64, rope_axes=(16, 24, 24), seed=5)
    m = b["packed_seq_params"]
    assert m.video_lens == [48, 16, 80] and m.caption_lens == [16, 8, 12]
    assert b["hidden_states"].shape[1] == sum(m.video_lens)
    # the same generator behind the fixed-shape helper: identical clips for identical seeds
    a1 = synthetic_packed_batch(2, (3, 8, 8), 8, text_dim=64, rope_axes=(16, 24, 24), seed=9)
    a2 = synthetic_items_batch([((3, 8, 8), True), ((3, 8, 8), False)], [8, 8], text_dim=64,
                               rope_axes=(16, 24, 24), seed=9)
    assert torch.equal(a1["hidden_states"], a2["hidden_states"])
    # a long single clip splits into strided CP shards that cover every video row once
    long = synthetic_items_batch([((9, 8, 8), True)], [16], text_dim=64, rope_axes=(16, 24, 24), seed=1)
    rows = 0
    for r in range(4):
        rows += strided_split(long, 4, r)["hidden_states"].shape[1]
    assert rows == long["hidden_states"].shape[1]


def test_loader_inputs_fail_fast(tmp_path):
    from pan2_b200.data.packing import CsvStream
    with pytest.raises(ValueError):
        CsvStream([])  # no video CSV files
    empty = tmp_path / "empty.csv"
    empty.write_text("latent_path,caption\n")
    with pytest.raises(ValueError, match="contain no rows"):
        next(iter(CsvStream([str(empty), str(empty)]).rows(None)))
    one = tmp_path / "one.csv"
    one.write_text("latent_path,caption\na.safetensors,hello\n")
    rows = CsvStream([str(empty), str(one)]).rows(None)
    first = [next(rows)[0]["caption"] for _ in range(3)]  # cycles through the non-empty file
    assert first == ["hello"] * 3


def test_image_stream_fails_fast_on_empty_tars(tmp_path, sample_dir):
    import tarfile
    from pan2_b200.data.packing import ImageCursor
    empty = tmp_path / "empty.tar"
    with tarfile.open(empty, "w"):
        pass
    ds = _dataset(sample_dir, image_tars=[str(empty), str(empty)])
    with pytest.raises(ValueError, match="no complete samples"):
        next(ds._image_stream(ImageCursor()))
    # an empty tar beside a real one: the stream keeps cycling through the real one's samples
    ds = _dataset(sample_dir, image_tars=[str(empty), str(sample_dir / "images.tar")])
    real = ds.tars.index(str(sample_dir / "images.tar"))
    it = ds._image_stream(ImageCursor())
    got = [next(it)[2] for _ in range(14)]
    assert {r.shard_index for r in got} == {real}
    first = got[0].cycle
    assert [r.sample_index for r in got[:7]] == list(range(6)) + [0] and got[6].cycle == first + 1
    # resuming past the last sample of the only real tar is not mistaken for an empty pass
    it = ds._image_stream(ImageCursor(real, 6, 0))
    assert next(it)[2].sample_index == 0


def test_loader_reiteration_stops_previous_producer(sample_dir):
    loader = PackedLoader(_dataset(sample_dir, image_prob=0.0), device="cpu", dtype=torch.float32, seed=0)
    next(iter(loader))
    first = loader._thread
    next(iter(loader))  # restarts: the first producer must end instead of filling its old queue forever
    first.join(timeout=10)
    assert not first.is_alive()
    loader.close()
    assert not loader._thread.is_alive()


def test_loader_surfaces_producer_errors():
    class Broken:
        def __iter__(self):
            raise OSError("disk gone")
            yield  # pragma: no cover
    loader = PackedLoader(Broken(), device="cpu")
    with pytest.raises(OSError, match="disk gone"):
        next(iter(loader))
    loader.close()


def test_resume_reads_buffered_images_by_byte_range(sample_dir, monkeypatch):
    import pan2_b200.data.packing as packing
    full = list(itertools.islice(iter(_dataset(sample_dir, image_prob=0.8)), 6))
    k = next(i for i, p in enumerate(full[:-1]) if any(r.modality == "image" for b in p.state.buffer_items for r in b))
    st = DataloaderState.from_json(full[k].state.to_json())
    refs = [r for b in st.buffer_items for r in b if r.modality == "image"]
    assert refs and all(r.tar_members is not None and len(r.tar_members) == 4 for r in refs)
    ds = _dataset(sample_dir, resume=st, image_prob=0.8)
    scans = []
    real = packing.iter_tar_samples
    monkeypatch.setattr(packing, "iter_tar_samples", lambda path: scans.append(path) or real(path))
    from pan2_b200.data.packing import _Bin
    bins = [_Bin(ds.budgets) for _ in range(ds.num_buffers)]
    ds._restore_bins(bins)
    assert scans == []  # restored from the recorded ranges, without scanning a tar
    restored = [it for b in bins for it in b.items if it.modality == "image"]
    assert len(restored) == len(refs)
    # the same samples as a scan of the tar gives
    by_idx = {idx: (raw, text) for idx, _, raw, text, _ in real(str(sample_dir / "images.tar"))}
    for it in restored:
        scanned = ds._image_item(*by_idx[it.ref.sample_index], it.ref)
        assert torch.equal(it.latent, scanned.latent) and it.caption.text == scanned.caption.text


def test_tar_paths_expand_recursively_and_deduplicate(tmp_path):
    from pan2_b200.data.packing import expand_tar_paths
    (tmp_path / "a" / "b").mkdir(parents=True)
    for rel in ("a/x.tar", "a/b/y.tar", "z.tar"):
        (tmp_path / rel).write_bytes(b"")
    listing = tmp_path / "list.txt"
    listing.write_text(f"{tmp_path / 'a'}\n{tmp_path / 'z.tar'}\n\n")
    got = expand_tar_paths([str(tmp_path / "a"), str(listing), str(tmp_path / "a" / "x.tar")])
    assert got == sorted({str(tmp_path / p) for p in ("a/x.tar", "a/b/y.tar", "z.tar")})
    with pytest.raises(ValueError, match="neither"):
        expand_tar_paths([str(tmp_path / "missing")])


def test_tar_samples_from_a_start_index_plain_and_compressed(sample_dir, tmp_path):
    import gzip
    import shutil
    from pan2_b200.data.items import iter_tar_samples, read_tar_sample
    plain = str(sample_dir / "images.tar")
    gz = str(tmp_path / "images.tar.gz")
    with open(plain, "rb") as src, gzip.open(gz, "wb") as dst:
        shutil.copyfileobj(src, dst)
    every = list(iter_tar_samples(plain))
    assert [s[0] for s in every] == list(range(6)) and all(s[4] is not None for s in every)
    tail = list(iter_tar_samples(plain, start=4))
    assert [(s[0], s[2], s[3]) for s in tail] == [(s[0], s[2], s[3]) for s in every[4:]]
    assert read_tar_sample(plain, every[3][4]) == (every[3][2], every[3][3])
    zipped = list(iter_tar_samples(gz, start=2))
    assert [(s[0], s[2], s[3]) for s in zipped] == [(s[0], s[2], s[3]) for s in every[2:]]
    assert all(s[4] is None for s in zipped)  # no byte ranges inside a compressed stream


def test_task_draws_follow_the_reference_ranges():
    from pan2_b200.data.items import ItemRef, draw_task
    refs = [ItemRef(global_index=i, local_index=i, local_file_pos=100 * i) for i in range(200)]
    cont = [draw_task(3, r, 21, 1.0, 0.0, 0.0)[0] for r in refs]
    assert min(cont) == 1 and max(cont) == 10  # 1 .. T // 2
    assert {draw_task(3, r, 21, 0.0, 1.0, 0.0)[0] for r in refs} == {1}
    assert {draw_task(3, r, 1, 0.5, 0.5, 0.0)[0] for r in refs} == {0}  # one latent frame: no prefix
    drops = [draw_task(3, r, 21, 0.0, 0.0, 0.3)[1] for r in refs]
    assert 0.15 < sum(drops) / len(drops) < 0.45
    assert draw_task(3, refs[7], 21, 0.4, 0.3, 0.1) == draw_task(3, refs[7], 21, 0.4, 0.3, 0.1)


def test_caption_with_lone_surrogates_is_cleaned(sample_dir):
    ds = _dataset(sample_dir)
    row, ref = next(ds.stream.rows(None))
    row = dict(row, caption="a cat \ud83d sits")
    it = ds._video_item((row, ref))
    assert it is not None and it.caption.text == "a cat  sits"


def test_dynamic_shift_sees_pixels_and_frames_of_the_token_grid(sample_dir):
    from pan2_b200.diffusion.flow_matching import shift_timesteps
    loader = PackedLoader(_dataset(sample_dir), device="cpu", shift_mode="dynamic")
    assert {k: loader.shift_kwargs[k] for k in ("frame_stride", "pixel_stride_h", "pixel_stride_w")} == \
        {"frame_stride": 4, "pixel_stride_h": 32, "pixel_stride_w": 32}
    t = torch.tensor([300.0, 700.0])
    # a 704 x 1280, 81-frame clip: token grid (21, 22, 40) at patch (1, 2, 2) == latent grid (21, 44, 80)
    tok = shift_timesteps(t, 1000, mode="dynamic", latent_shapes=torch.tensor([[21.0, 22, 40]] * 2),
                          **{k: loader.shift_kwargs[k] for k in ("frame_stride", "pixel_stride_h", "pixel_stride_w")})
    lat = shift_timesteps(t, 1000, mode="dynamic", latent_shapes=torch.tensor([[21.0, 44, 80]] * 2))
    assert torch.allclose(tok, lat)
    area, frames = 704 * 1280, 81
    s = math.exp(0.5 * ((1.15 - 0.5) / (1024 ** 2 - 256 ** 2) * (area - 256 ** 2) + 0.5 + 1.64 / 120 * (frames - 1)))
    f = t / 1000
    assert torch.allclose(tok, s * f / (1 + (s - 1) * f) * 1000, rtol=1e-5)


def test_timesteps_are_rounded_to_the_batch_dtype(sample_dir):
    ds = _dataset(sample_dir, image_prob=0.0)
    for dtype in (torch.bfloat16, torch.float32):
        loader = PackedLoader(ds, device="cpu", dtype=dtype, seed=0, shift=3.0)
        batch, _ = next(iter(loader))
        loader.close()
        t = batch["timestep"]
        assert t.dtype == torch.float32 and torch.equal(t, t.to(dtype).float())
