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
