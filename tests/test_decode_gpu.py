"""GPU parity of the fused LZ4 decode + recombine and of the plane recombine,
bit-exact against the oracle (liblz4 + the restated decoder) and the golden
fixtures."""
import os

import numpy as np
import pytest
import torch

from oracle import codec

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "codec_cases.npz")


def _ops():
    from zmoe import ops
    return ops


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _fixture_cases():
    g = np.load(GOLD)
    for key in g["names"]:
        key = str(key)
        bits = g[key.split("__")[0] + "__bits"]
        csz = [int(v) for v in g[key + "__csz"]]
        osz = [int(v) for v in g[key + "__osz"]]
        raw = g[key + "__blocks"].tobytes()
        blocks, pos = [], 0
        for c in csz:
            blocks.append(raw[pos:pos + c])
            pos += c
        yield key, bits, blocks, osz


def test_decode_matches_golden_fixtures():
    ops = _ops()
    for key, bits, blocks, osz in _fixture_cases():
        _, sm = codec.split_planes(bits)
        ct = ops.CompressedTensor(blocks, osz, sm.tobytes())
        out, st = ct.decode()
        torch.cuda.synchronize()
        assert (st.cpu().numpy() == 0).all(), (key, st.cpu().numpy())
        assert np.array_equal(_bits(out), bits), key


@pytest.mark.parametrize("std", [0.005, 0.02, 0.08])
@pytest.mark.parametrize("codec_name", ["LZ4HC", "LZ4"])
def test_decode_full_qwen_expert_matrix(std, codec_name):
    ops = _ops()
    gen = torch.Generator().manual_seed(0)
    w = (torch.randn(1408, 2048, generator=gen) * std).to(torch.bfloat16)
    bits = codec.bf16_bits(w)
    blocks, osz, sm = codec.encode_tensor(bits, 3, codec_name)
    assert osz == [961195, 961195, 961194]
    ct = ops.CompressedTensor(blocks, osz, sm.tobytes())
    out, st = ct.decode()
    torch.cuda.synchronize()
    assert (st.cpu().numpy() == 0).all()
    assert np.array_equal(_bits(out), bits)


def test_decode_many_chunks_one_launch_unaligned_destinations():
    ops = _ops()
    gen = torch.Generator().manual_seed(3)
    mats = [(torch.randn(97, 531, generator=gen) * 0.03).to(torch.bfloat16) for _ in range(11)]
    cts, bits_all = [], []
    for m in mats:
        bits = codec.bf16_bits(m)
        blocks, osz, sm = codec.encode_tensor(bits, 5)
        cts.append(ops.CompressedTensor(blocks, osz, sm.tobytes()))
        bits_all.append(bits)
    total = sum(b.size for b in bits_all)
    dst = torch.zeros(total + 3, dtype=torch.bfloat16, device="cuda")
    descs, pos = [], 1                       # odd element offset: unaligned output
    views = []
    for ct, b in zip(cts, bits_all):
        v = dst[pos:pos + b.size]
        descs.extend(ct.descs(v))
        views.append(v)
        pos += b.size
    scratch = ops.map_scratch([d[4] for d in descs], "cuda")
    table = ops.chunk_table(descs, "cuda", scratch)
    st = ops.decode_chunks(table, len(descs))
    torch.cuda.synchronize()
    assert (st.cpu().numpy() == 0).all()
    for v, b in zip(views, bits_all):
        assert np.array_equal(_bits(v), b)
    assert _bits(dst[:1])[0] == 0 and (_bits(dst[pos:]) == 0).all()   # nothing written outside


def test_decode_long_runs_and_overlapping_matches():
    ops = _ops()
    # long literal runs (incompressible), long matches (constant runs, offset 1)
    rng = np.random.default_rng(5)
    parts = [rng.integers(0, 65536, 3000, dtype=np.uint16), np.full(70000, 0x3C00, np.uint16),
             rng.integers(0, 65536, 77, dtype=np.uint16), np.tile(np.arange(3, dtype=np.uint16) + 0x3F00, 9000)]
    bits = np.concatenate(parts)
    for chunks, indexed in ((1, True), (2, True), (7, True), (2, False)):
        blocks, osz, sm = codec.encode_tensor(bits, chunks)
        out, st = ops.CompressedTensor(blocks, osz, sm.tobytes(), indexed=indexed).decode()
        torch.cuda.synchronize()
        assert (st.cpu().numpy() == 0).all()
        assert np.array_equal(_bits(out), bits)


def test_decode_reports_malformed_blocks_without_trapping():
    ops = _ops()
    gen = torch.Generator().manual_seed(9)
    bits = codec.bf16_bits((torch.randn(64, 300, generator=gen) * 0.02).to(torch.bfloat16))
    blocks, osz, sm = codec.encode_tensor(bits, 1)
    blk = blocks[0]
    seqs = codec.lz4_sequences(blk)
    # (a) truncated block: lengths run past the end, or the block ends short
    trunc = blk[: len(blk) // 2]
    # (b) a zero offset in the first sequence that has a match
    s0 = next(s for s in seqs if s[4] > 0)
    off_pos = s0[0] + 1 + (1 if s0[2] >= 15 else 0) + s0[2]
    zero = bytearray(blk)
    zero[off_pos:off_pos + 2] = b"\0\0"
    # (c) an offset reaching before the chunk start
    far = bytearray(blk)
    far[off_pos:off_pos + 2] = (min(65535, s0[1] + s0[2] + 1)).to_bytes(2, "little")
    # (d) the block describes fewer bytes than original_size
    cases = {"trunc": (trunc, osz[0]), "zero_off": (bytes(zero), osz[0]),
             "far_off": (bytes(far), osz[0]), "short": (blk, osz[0] + 100)}
    sm_pad = np.concatenate([sm, np.zeros(100, np.uint8)])
    expect = {"zero_off": 1, "far_off": 1, "short": 3}
    for name, (b, o) in cases.items():
        if name != "short":
            with pytest.raises(ValueError):       # the host index walk rejects it
                ops.build_index(b, o)
        ct = ops.CompressedTensor([b], [o], sm_pad[:o].tobytes(), indexed=False)
        _, st = ct.decode()
        torch.cuda.synchronize()
        code = int(st.cpu()[0])
        assert code != 0, name
        if name in expect:
            assert code == expect[name], (name, code)
        rc, _ = codec.lz4_decompress_restated(b, o)
        assert rc < 0 or rc < o, name           # the oracle rejects it too
    # the context is still usable afterwards
    out, st = ops.CompressedTensor(blocks, osz, sm.tobytes()).decode()
    torch.cuda.synchronize()
    assert int(st.cpu()[0]) == 0 and np.array_equal(_bits(out), bits)


@pytest.mark.parametrize("n,offset", [(1, 0), (15, 0), (16, 0), (4099, 0), (1 << 20, 0), (1000, 3), (65536 + 7, 1)])
def test_tensor_recover_bit_exact(n, offset):
    ops = _ops()
    rng = np.random.default_rng(n)
    bits = rng.integers(0, 65536, n, dtype=np.uint16)
    exp, sm = codec.split_planes(bits)
    e = torch.zeros(n + offset, dtype=torch.uint8, device="cuda")
    s = torch.zeros(n + offset, dtype=torch.uint8, device="cuda")
    e[offset:] = torch.from_numpy(exp).cuda()
    s[offset:] = torch.from_numpy(sm).cuda()
    out = ops.tensor_recover(e[offset:], s[offset:])
    torch.cuda.synchronize()
    assert np.array_equal(_bits(out), bits)


@pytest.mark.parametrize("indexed", [True, False])
def test_decode_indexed_and_unindexed(indexed):
    """With the slice index 4 warps map sources in parallel; without it one
    warp decodes serially; both must give the same bytes."""
    ops = _ops()
    gen = torch.Generator().manual_seed(21)
    w = (torch.randn(512, 2048, generator=gen) * 0.02).to(torch.bfloat16)
    bits = codec.bf16_bits(w)
    blocks, osz, sm = codec.encode_tensor(bits, 3)
    ct = ops.CompressedTensor(blocks, osz, sm.tobytes(), indexed=indexed)
    out, st = ct.decode()
    torch.cuda.synchronize()
    assert (st.cpu().numpy() == 0).all(), st.cpu().numpy()
    assert np.array_equal(_bits(out), bits)


def test_decode_small_offsets_across_segments():
    """Periodic data gives short offsets that reach into the previous segment."""
    ops = _ops()
    rng = np.random.default_rng(8)
    base = rng.integers(0, 65536, 37, dtype=np.uint16)
    bits = np.concatenate([np.tile(base, 3000), rng.integers(0, 65536, 5000, dtype=np.uint16),
                           np.tile(base[:5], 20000)])
    blocks, osz, sm = codec.encode_tensor(bits, 1)
    for indexed in (True, False):
        out, st = ops.CompressedTensor(blocks, osz, sm.tobytes(), indexed=indexed).decode()
        torch.cuda.synchronize()
        assert (st.cpu().numpy() == 0).all()
        assert np.array_equal(_bits(out), bits)


def test_decode_index_of_another_block_is_reported_not_trapped():
    """An index that does not belong to the block (the host builds it at load
    time, so this is a caller error) must end in a status word or in the right
    bytes, never in a fault; the context stays usable."""
    ops = _ops()
    gen = torch.Generator().manual_seed(31)
    a = codec.bf16_bits((torch.randn(300, 700, generator=gen) * 0.02).to(torch.bfloat16))
    b = codec.bf16_bits((torch.randn(300, 700, generator=gen) * 0.07).to(torch.bfloat16))
    ba, oa, sma = codec.encode_tensor(a, 1)
    bb, ob, smb = codec.encode_tensor(b, 1)
    assert oa == ob
    ct = ops.CompressedTensor(bb, ob, smb.tobytes())
    ct.indexes = ops.CompressedTensor(ba, oa, sma.tobytes()).indexes.clone()
    ct.index_rows = [int(ct.indexes.shape[0])]
    out, st = ct.decode()
    torch.cuda.synchronize()
    code = int(st.cpu()[0])
    assert code != 0 or np.array_equal(_bits(out), b)
    out, st = ops.CompressedTensor(ba, oa, sma.tobytes()).decode()
    torch.cuda.synchronize()
    assert int(st.cpu()[0]) == 0 and np.array_equal(_bits(out), a)
