"""The `ZipMoE` drop-in on the GPU, driven the way the reference drives it:
offload experts to the reference file format, register them with the
expert_dispatcher, run experts/expert_executor.py's dispatch_local sequence and
compare every expert output with the oracle FFN."""
import pytest
import torch

from oracle import moe
from zipmoe_flow import dispatch_local, make_handle, split_exp_chunks

pytestmark = pytest.mark.gpu


def _setup(tmp_path, kind=0, E=6, H=256, I=96, layers=2, topk=2, cache_ratio=0.0, policy="LFU"):
    import ZipMoE
    g = torch.Generator().manual_seed(4)
    per = 3 if kind == 0 else 2
    shapes = [(I, H), (I, H), (H, I)] if kind == 0 else [(I, H), (H, I)]
    w = [[[(torch.randn(*s, generator=g) * 0.05).to(torch.bfloat16) for s in shapes] for _ in range(E)]
         for _ in range(layers)]
    h = make_handle(ZipMoE, str(tmp_path), E, layers, per, H * I, topk, cache_ratio=cache_ratio, policy=policy)
    ids, tensors, chunks, sms = [], [], [], []
    tid = 100
    id_of = {}
    for l in range(layers):
        for e in range(E):
            id_of[(l, e)] = []
            for t in w[l][e]:
                c, s = split_exp_chunks(t, 3)
                ids.append(tid); tensors.append(t); chunks.append(c); sms.append(s)
                id_of[(l, e)].append(tid)
                tid += 1
    h.batch_offload(ids, tensors, chunks, sms)
    h.open_offload_file()
    d = ZipMoE.expert_dispatcher(E, layers, kind, 0)
    for (l, e), tids in id_of.items():
        d.register_expert(l, e, tids)
    return ZipMoE, h, d, w, id_of


def _mask(T, E, topk, seed):
    g = torch.Generator().manual_seed(seed)
    m = torch.zeros(T, E, dtype=torch.int64)
    for t in range(T):
        m[t, torch.randperm(E, generator=g)[:topk]] = 1
    return m


def _check(res, x, mask, w, layer, kind):
    assert len(res) == int((mask.sum(0) > 0).sum())
    for out, l, e, hit in res:
        assert l == layer and hit in (0, 1)
        tok = torch.nonzero(mask[:, e]).flatten()
        f = moe.swiglu_fp32 if kind == 0 else moe.relu_ffn_fp32
        ref = f(x[tok].cpu(), *w[layer][e])
        assert out.dtype == torch.bfloat16 and out.shape == ref.shape and out.is_cuda
        d = (out.float().cpu() - ref).abs()
        assert d.max() <= 2e-2 and d.mean() / ref.abs().mean() <= 5e-3, (e, float(d.max()))


@pytest.mark.parametrize("kind", [0, 1])
def test_dispatch_local_matches_oracle(tmp_path, kind):
    Z, h, d, w, _ = _setup(tmp_path, kind=kind)
    T, E = 40, 6
    for layer, seed in ((0, 1), (1, 2), (0, 3)):
        x = (torch.randn(T, 256, generator=torch.Generator().manual_seed(seed))).to(torch.bfloat16).cuda()
        mask = _mask(T, E, 2 if kind == 0 else 1, seed)
        res = dispatch_local(d, x, mask.cuda(), layer)
        _check(res, x, mask, w, layer, kind)


def test_prefetch_makes_hits_and_obtain_tensor_is_exact(tmp_path):
    Z, h, d, w, id_of = _setup(tmp_path, cache_ratio=1.0, policy="ZipMoE")
    for e in range(3):
        got = d.obtain_tensor(1, e, 2)
        assert torch.equal(got.cpu().view(torch.int16), w[1][e][2].view(torch.int16))
    d.submit_prefetch(0, 4, 1.0)
    d.enqueue_prefetch(0, 5)
    T = 16
    x = torch.randn(T, 256, generator=torch.Generator().manual_seed(9)).to(torch.bfloat16).cuda()
    mask = torch.zeros(T, 6, dtype=torch.int64)
    mask[:8, 4] = 1
    mask[8:, 5] = 1
    mask[::3, 1] = 1
    res = dispatch_local(d, x, mask.cuda(), 0)
    hits = {e: hit for _, _, e, hit in res}
    assert hits[4] == 1 and hits[5] == 1 and hits[1] == 0
    _check(res, x, mask, w, 0, 0)
    h.reset_access_counts()


def test_begin_end_materialise_registered_tensor(tmp_path):
    Z, h, d, w, id_of = _setup(tmp_path, layers=1)
    p = torch.nn.Parameter(torch.zeros(1, dtype=torch.bfloat16), requires_grad=False)
    tid = id_of[(0, 2)][1]
    h.register(p.data, tid)
    assert h.begin(0, p) == tid
    assert p.is_cuda and torch.equal(p.data.cpu().view(torch.int16), w[0][2][1].view(torch.int16))
    h.end(0, p)
    assert p.numel() == 1 and not p.is_cuda
    assert h.get_node_default_device([tid]) == torch.cuda.current_device()


def test_batch_offload_with_gpu_encoder(tmp_path):
    """set_gpu_encode(True): batch_offload encodes every LZ4HC chunk of the
    batch on the GPU.  The file keeps the reference's layout; each block is
    the oracle's statement of the GPU parse byte for byte, liblz4 restores it,
    and begin() materialises every tensor exactly."""
    import numpy as np
    import ZipMoE
    from oracle import codec, fmt
    g = torch.Generator().manual_seed(9)
    ts = [(torch.randn(96, 256, generator=g) * 0.05).to(torch.bfloat16) for _ in range(6)]
    h = make_handle(ZipMoE, str(tmp_path), 2, 1, 3, 96 * 256, 1)
    h.set_gpu_encode(True)
    ids = list(range(200, 206))
    chunks, sms = zip(*[split_exp_chunks(t, 3) for t in ts])
    h.batch_offload(ids, ts, list(chunks), list(sms))
    h.open_offload_file()
    metas = fmt.deserialize_index((tmp_path / "zipmoe_index").read_bytes())
    raw = (tmp_path / "zipmoe_param").read_bytes()
    for tid, t, cs in zip(ids, ts, chunks):
        m = metas[tid]
        for c, off, csz, osz in zip(cs, m.exp_file_offsets, m.compressed_sizes, m.original_sizes):
            blk = raw[off:off + csz]
            c = np.ascontiguousarray(c, dtype=np.uint8)
            assert osz == c.size and blk == codec.lz4_encode_chains(c, 256)
            assert np.array_equal(codec.lz4_decompress(blk, osz), c)
        p = torch.nn.Parameter(torch.zeros(1, dtype=torch.bfloat16), requires_grad=False)
        h.register(p.data, tid)
        assert h.begin(0, p) == tid
        assert torch.equal(p.data.cpu().view(torch.int16), t.view(torch.int16))
        h.end(0, p)
