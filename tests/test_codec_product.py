"""The product's offload encoder (libzmoe.so) against the oracle codec."""
import numpy as np
import torch

from oracle import codec as ocodec


def test_split_planes_matches_oracle():
    from zmoe import codec
    rng = np.random.default_rng(1)
    bits = rng.integers(0, 65536, 100003, dtype=np.uint16)
    e1, s1 = codec.split_planes(bits)
    e2, s2 = ocodec.split_planes(bits)
    assert np.array_equal(e1, e2) and np.array_equal(s1, s2)


def test_encode_matches_oracle_bytes_and_roundtrips():
    from zmoe import codec
    gen = torch.Generator().manual_seed(0)
    ts = [(torch.randn(64, 300, generator=gen) * 0.02).to(torch.bfloat16), torch.zeros(7, 9, dtype=torch.bfloat16)]
    for cod, lvl in (("LZ4HC", 9), ("LZ4", 5)):
        enc = codec.encode_tensors(ts, num_file_chunks=3, codec=cod, level=lvl, threads=2)
        for t, e in zip(ts, enc):
            bits = ocodec.bf16_bits(t)
            blocks, osz, sm = ocodec.encode_tensor(bits, 3, cod, lvl, lvl)
            assert e.blocks == blocks and e.original_sizes == osz and e.sm == sm.tobytes()
            assert np.array_equal(ocodec.decode_tensor(e.blocks, e.original_sizes, np.frombuffer(e.sm, np.uint8)), bits)


def test_slice_index_matches_token_walk():
    """Entry j names the sequence that contains output byte j * slice."""
    from zmoe import ops
    gen = torch.Generator().manual_seed(4)
    bits = ocodec.bf16_bits((torch.randn(100, 700, generator=gen) * 0.02).to(torch.bfloat16))
    bits = np.concatenate([bits, np.full(5000, 0x3C00, np.uint16)])     # a long run too
    blocks, osz, _ = ocodec.encode_tensor(bits, 2)
    for blk, o in zip(blocks, osz):
        seqs = ocodec.lz4_sequences(blk)
        for seg in (256, 4096):
            idx = ops.build_index(blk, o, seg)
            assert len(idx) == (o + seg - 1) // seg
            for j, (ip, op) in enumerate(idx.tolist()):
                b = j * seg
                want = next((s[0], s[1]) for s in seqs if s[1] <= b < s[1] + s[2] + s[4])
                assert (ip, op) == want, (seg, j)


def test_segment_index_rejects_malformed():
    from zmoe import ops
    import pytest
    exp = (np.arange(5000) % 7).astype(np.uint8)
    blk = ocodec.lz4_compress_hc(exp)
    with pytest.raises(ValueError):
        ops.build_index(blk[: len(blk) // 2], exp.size)
