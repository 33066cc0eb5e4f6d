"""Host logic on the CPU: BatchNorm fold, GLU row interleave, int8 quantisation, frame-grid chunk planning and the
per-rank shard plan (2 gloo ranks), and the op schemas / fake implementations used by torch.compile."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from granite_conv_b200 import dispatch, synth
from granite_conv_b200.weights import (fold_conv_bn_, glu_deinterleave, glu_interleave, prepare_from_params,
                                       quantize_per_channel)
from oracle import conv_module as O


class _RefLikeConvModule(nn.Module):
    """Attribute layout of the reference ConformerConvModule (conformer.py:161-173), for host-side tests."""

    def __init__(self, d=64, inner=128, k=15):
        super().__init__()
        self.norm = nn.LayerNorm(d)
        self.up_conv = nn.Conv1d(d, 2 * inner, 1)
        self.glu = nn.GLU(dim=1)
        self.depth_conv = nn.Module()
        self.depth_conv.conv = nn.Conv1d(inner, inner, k, groups=inner, bias=False, padding=k // 2)
        self.batch_norm = nn.BatchNorm1d(inner)
        self.down_conv = nn.Conv1d(inner, d, 1)


def test_fold_matches_oracle_and_is_idempotent():
    torch.manual_seed(0)
    m = _RefLikeConvModule()
    with torch.no_grad():
        m.batch_norm.running_mean.normal_(0, 0.1)
        m.batch_norm.running_var.uniform_(0.5, 1.5)
        m.batch_norm.weight.uniform_(0.8, 1.2)
        m.batch_norm.bias.normal_(0, 0.05)
    with pytest.raises(RuntimeError, match="eval"):
        fold_conv_bn_(m)
    m.eval()
    bn = m.batch_norm
    ow, ob = O.fold_bn(m.depth_conv.conv.weight.detach().numpy()[:, 0], bn.weight.detach().numpy(),
                       bn.bias.detach().numpy(), bn.running_mean.numpy(), bn.running_var.numpy(), bn.eps, False)
    x = torch.randn(2, 128, 40)
    before = m.batch_norm(m.depth_conv.conv(x))
    assert fold_conv_bn_(m) == 1
    assert isinstance(m.batch_norm, nn.Identity)
    np.testing.assert_array_equal(m.depth_conv.conv.weight.detach().numpy()[:, 0], ow)
    np.testing.assert_array_equal(m.depth_conv.conv.bias.detach().numpy(), ob)
    torch.testing.assert_close(m.depth_conv.conv(x), before, atol=1e-5, rtol=1e-5)
    assert fold_conv_bn_(m) == 0


def test_glu_interleave_layout():
    rows = torch.arange(512).reshape(512, 1)
    il = glu_interleave(rows)
    # block j of 256 rows = value rows [128j, 128j+128) then gate rows [256+128j, ...)
    assert il[:128, 0].tolist() == list(range(128))
    assert il[128:256, 0].tolist() == list(range(256, 384))
    assert il[256:384, 0].tolist() == list(range(128, 256))
    assert torch.equal(glu_deinterleave(il), rows)
    with pytest.raises(ValueError):
        glu_interleave(torch.zeros(100, 2))


def test_prepare_from_params_matches_oracle_bits():
    params = synth.make_params(1003)
    p = prepare_from_params(params, device="cpu", int8=True)
    prep = O.prepare_bf16(params)
    np.testing.assert_array_equal(p.dw_w.float().numpy(), prep["dw_w"])
    np.testing.assert_array_equal(p.dw_b.float().numpy(), prep["dw_b"])
    np.testing.assert_array_equal(glu_deinterleave(p.w1_glu).float().numpy(), prep["w1"])
    np.testing.assert_array_equal(glu_deinterleave(p.b1_glu).numpy(), prep["b1"])
    np.testing.assert_array_equal(p.w2.float().numpy(), prep["w2"])
    q1, s1 = O.quantize_per_channel(prep["w1"])
    np.testing.assert_array_equal(glu_deinterleave(p.w1q_glu).numpy(), q1)
    np.testing.assert_allclose(glu_deinterleave(p.s1_glu).numpy(), s1, rtol=1e-7)
    q, s = quantize_per_channel(torch.from_numpy(prep["w2"]))
    oq, _ = O.quantize_per_channel(prep["w2"])
    np.testing.assert_array_equal(q.numpy(), oq)


def test_bucket_and_chunks():
    assert dispatch.bucket_frames(1) == 128 and dispatch.bucket_frames(128) == 128
    assert dispatch.bucket_frames(129) == 256 and dispatch.bucket_frames(77, 0) == 77
    lens = synth.sample_lengths(1005, 512)
    assert lens.min() >= 64 and lens.max() <= 1536
    chunks = dispatch.plan_chunks(lens)
    assert sum(c.B for c in chunks) == 512
    assert all(c.B <= 48 for c in chunks)
    seen = np.concatenate([c.index for c in chunks])
    assert sorted(seen.tolist()) == list(range(512))
    for c in chunks:
        assert c.T % 128 == 0 and c.T >= c.lengths.max() and c.T - 128 < c.lengths.max()
        np.testing.assert_array_equal(c.lengths, lens[c.index])
    # logical batches of 128 split 48 + 48 + 32
    assert [c.B for c in chunks[:3]] == [48, 48, 32]
    # sorted by length: chunk maxima are non-decreasing
    mx = [int(c.lengths.max()) for c in chunks]
    assert mx == sorted(mx)
    assert dispatch.plan_chunks([]) == []
    with pytest.raises(ValueError):
        dispatch.plan_chunks([-1])


def test_shard_balance():
    chunks = dispatch.plan_chunks(synth.sample_lengths(1005, 512))
    for world in (1, 2, 4, 8):
        shards = dispatch.shard_chunks(chunks, world)
        ids = sorted(int(i) for s in shards for c in s.chunks for i in c.index)
        assert ids == list(range(512))
        loads = [s.padded_frames for s in shards]
        assert max(loads) - min(loads) <= max(c.padded_frames for c in chunks)


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    chunks = dispatch.plan_chunks(synth.sample_lengths(1005, 512))
    mine = dispatch.shard_chunks(chunks, world)[rank]
    n_mine = sum(c.B for c in mine.chunks)
    ids = torch.tensor(sorted(int(i) for c in mine.chunks for i in c.index) + [-1] * (512 - n_mine))
    gathered = [torch.empty_like(ids) for _ in range(world)]
    dist.all_gather(gathered, ids)
    load = torch.tensor([mine.padded_frames], dtype=torch.int64)
    loads = [torch.empty_like(load) for _ in range(world)]
    dist.all_gather(loads, load)
    # the utterance split: each rank plans chunks from its own share of the sorted utterances
    lens = synth.sample_lengths(1005, 512)
    share = dispatch.shard_utterances(lens, world)[rank]
    own = dispatch.plan_chunks(lens[share])
    uids = torch.tensor(sorted(int(share[i]) for c in own for i in c.index) + [-1] * (512 - share.size))
    ugathered = [torch.empty_like(uids) for _ in range(world)]
    dist.all_gather(ugathered, uids)
    tiles = torch.tensor([sum(-(-int(L) // 128) for c in own for L in c.lengths)], dtype=torch.int64)
    tgathered = [torch.empty_like(tiles) for _ in range(world)]
    dist.all_gather(tgathered, tiles)
    if rank == 0:
        allids = sorted(int(v) for g in gathered for v in g.tolist() if v >= 0)
        uall = sorted(int(v) for g in ugathered for v in g.tolist() if v >= 0)
        q.put((allids, [int(v.item()) for v in loads], uall, [int(v.item()) for v in tgathered]))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_shards_cover_every_utterance_once():
    """Two gloo ranks each compute the shard plan locally (no exchange needed) and together cover every
    utterance exactly once with balanced padded work."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 2000)
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    allids, loads, uall, tiles = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert allids == list(range(512))
    assert abs(loads[0] - loads[1]) <= 48 * 1536
    assert uall == list(range(512))                      # utterance split: every utterance once
    assert max(tiles) <= 1.02 * sum(tiles) / 2           # and the 128-row tiles of work balance within 2 %


def test_shard_utterances_balance():
    """Sorted utterances dealt round robin: every utterance exactly once at every world size, and the busiest rank's
    128-row tiles within 2 % of the mean at 8 ranks (whole chunks dealt greedily reach only ~1.24x there)."""
    lens = synth.sample_lengths(1005, 512)
    for world in (1, 2, 4, 8):
        shares = dispatch.shard_utterances(lens, world)
        assert sorted(int(i) for s in shares for i in s) == list(range(512))
        tiles = [sum(-(-int(L) // 128) for L in lens[s]) for s in shares]
        assert max(tiles) <= 1.02 * sum(tiles) / world, (world, tiles)
    with pytest.raises(ValueError):
        dispatch.shard_utterances(lens, 0)


def test_op_schemas_and_fakes():
    import granite_conv_b200.ops  # noqa: F401
    from torch._subclasses.fake_tensor import FakeTensorMode
    assert "dwconv_silu(Tensor x, Tensor weight, Tensor bias) -> Tensor" in str(
        torch.ops.granite.dwconv_silu.default._schema)
    assert "dwconv_silu_glu(Tensor x2, Tensor weight, Tensor bias) -> Tensor" in str(
        torch.ops.granite.dwconv_silu_glu.default._schema)
    with FakeTensorMode(allow_non_fake_inputs=False):
        cl = torch.empty(2, 37, 256, dtype=torch.bfloat16, device="meta").transpose(1, 2)
        w = torch.empty(256, 1, 15, dtype=torch.bfloat16, device="meta")
        b = torch.empty(256, dtype=torch.bfloat16, device="meta")
        y = torch.ops.granite.dwconv_silu(cl, w, b)
        assert y.shape == (2, 256, 37) and y.stride() == (37 * 256, 1, 256)
        cf = torch.empty(2, 256, 37, dtype=torch.bfloat16, device="meta")
        assert torch.ops.granite.dwconv_silu(cf, w, b).stride() == (256 * 37, 37, 1)
        x2 = torch.empty(2, 37, 512, dtype=torch.bfloat16, device="meta").transpose(1, 2)
        y2 = torch.ops.granite.dwconv_silu_glu(x2, w, b)
        assert y2.shape == (2, 256, 37) and y2.stride() == (37 * 256, 1, 256)
