"""The `ZipMoE` drop-in module: offload files byte-identical to the
reference's format (restated in oracle/fmt.py), index round trips, method
surface of csrc/binding/bindings.cpp:17-222.  No GPU needed."""
import os

import numpy as np
import pytest
import torch

from oracle import codec as oc
from oracle import fmt
from zipmoe_flow import make_handle, split_exp_chunks

HANDLE_METHODS = ["open_offload_file", "offload", "batch_offload", "register", "begin", "end", "set_topology",
                  "update_tensor_map", "is_tensor_offloaded", "is_tensor_index_initialized",
                  "get_node_default_device", "fetch_tensors", "reset_access_counts"]
DISPATCHER_METHODS = ["register_expert", "obtain_tensor", "enqueue_expert", "enqueue_prefetch", "submit_prefetch",
                      "ops_schedule", "set_inputs", "set_expected_queue", "wait_expert"]


def _mod():
    import ZipMoE
    return ZipMoE


def test_method_surface():
    Z = _mod()
    for m in HANDLE_METHODS:
        assert hasattr(Z.zipmoe_prefetch_handle, m), m
    for m in DISPATCHER_METHODS:
        assert hasattr(Z.expert_dispatcher, m), m


def _tensors(seed=3):
    g = torch.Generator().manual_seed(seed)
    return [(torch.randn(96, 256, generator=g) * 0.02).to(torch.bfloat16),
            (torch.randn(96, 256, generator=g) * 0.05).to(torch.bfloat16),
            (torch.randn(256, 96, generator=g) * 0.02).to(torch.bfloat16)]


@pytest.mark.parametrize("code", ["LZ4HC", "LZ4"])
def test_offload_files_match_reference_format(tmp_path, code):
    Z = _mod()
    ts = _tensors()
    dense = (torch.randn(7, 33, generator=torch.Generator().manual_seed(1)) * 3).to(torch.bfloat16)
    h = make_handle(Z, str(tmp_path), 1, 1, 3, 96 * 256, 2, code=code)
    assert not h.is_tensor_index_initialized()
    c0, s0 = split_exp_chunks(ts[0], 3)
    h.offload(5, ts[0], c0, s0, True)
    h.offload(9, dense, [], np.zeros(0, np.uint8), False)
    rest = [split_exp_chunks(t, 3) for t in ts[1:]]
    h.batch_offload([11, 12], ts[1:], [r[0] for r in rest], [r[1] for r in rest])
    assert h.is_tensor_offloaded(11) and not h.is_tensor_offloaded(13)
    # the same bytes through the format restatement and liblz4
    w = fmt.ParamWriter()
    metas = {}
    for tid, t in ((5, ts[0]),):
        blocks, osz, sm = oc.encode_tensor(oc.bf16_bits(t), 3, code, 9 if code == "LZ4HC" else 5)
        metas[tid] = w.offload_sparse(tid, list(t.shape), blocks, osz, sm.tobytes())
    metas[9] = w.offload_dense(9, list(dense.shape), dense.view(torch.int16).numpy().tobytes(), 3)
    for tid, t in ((11, ts[1]), (12, ts[2])):
        blocks, osz, sm = oc.encode_tensor(oc.bf16_bits(t), 3, code, 9 if code == "LZ4HC" else 5)
        metas[tid] = w.offload_sparse(tid, list(t.shape), blocks, osz, sm.tobytes())
    assert open(tmp_path / "zipmoe_param", "rb").read() == bytes(w.buf)
    assert open(tmp_path / "zipmoe_index", "rb").read() == fmt.serialize_index(metas)
    with pytest.raises(RuntimeError, match="offloaded twice"):
        h.offload(5, ts[0], c0, s0, True)


def test_reads_index_written_by_the_format_restatement(tmp_path):
    Z = _mod()
    t = _tensors(7)[0]
    blocks, osz, sm = oc.encode_tensor(oc.bf16_bits(t), 3, "LZ4HC", 9)
    w = fmt.ParamWriter()
    metas = {42: w.offload_sparse(42, list(t.shape), blocks, osz, sm.tobytes())}
    (tmp_path / "zipmoe_param").write_bytes(bytes(w.buf))
    (tmp_path / "zipmoe_index").write_bytes(fmt.serialize_index(metas))
    h = make_handle(Z, str(tmp_path), 1, 1, 3, t.numel(), 2)
    assert h.is_tensor_index_initialized() and h.is_tensor_offloaded(42)
    h.open_offload_file()


def test_rejections(tmp_path):
    Z = _mod()
    with pytest.raises(RuntimeError, match="CODE_TYPE"):
        make_handle(Z, str(tmp_path / "a"), 1, 1, 3, 10, 1, code="ZSTD")
    h = make_handle(Z, str(tmp_path / "b"), 1, 1, 3, 96 * 256, 2)
    t = _tensors()[0]
    c, s = split_exp_chunks(t, 3)
    with pytest.raises(RuntimeError, match="num_file_chunks"):
        h.offload(1, t, c[:2], s, True)
    with pytest.raises(RuntimeError, match="num_elements"):
        h.offload(2, t, c, s[:-1], True)
    with pytest.raises(RuntimeError, match="dtype"):
        Z.expert_dispatcher(4, 1, 0, 1)
