"""Generate the committed golden fixtures under tests/golden/.

Run in a container that has the reference checkout (it is read, never
modified):

    python tests/golden/make_golden.py <path of the reference checkout>

Fixtures:

* ``codec_cases.npz`` — small BF16 tensors (seeded normal, all-zero, constant,
  ragged sizes, tiny sizes, random bit patterns), their exponent / sign+mantissa
  planes, their LZ4HC-9 and LZ4-fast chunk blocks produced by liblz4 (the
  reference codec library), and the bytes liblz4 decodes them back to.
* ``qwen_block_c2.npz`` — the same for the reference's Qwen block at the full
  Qwen1.5-MoE-A2.7B layer shape with the benchmark's seeded weights (64 tokens).
* ``qwen_block.npz`` / ``deepseek_block.npz`` — inputs are regenerated from
  seeds by the tests; the fixture holds the outputs of the reference's own
  ``customized/qwen.py`` Qwen2MoEBlock and ``customized/deepseek.py``
  DeepseekMoEBlock (with the ``MoEGate`` / ``DeepseekV2MLP`` classes of
  ``models/deepseek/modeling_deepseek.py``).  Their expert dispatcher is
  replaced by a CPU stand-in that runs each expert module on its gathered
  tokens, which is what ``ExpertDispatcher::GPUExecFunc`` computes
  (``csrc/dispatcher/expert_module.cpp:39-50``), returning results in expert
  order.
* ``predictor_cases.json`` — the reference ExpertPredictor's predictions on a
  seeded replay.
* ``cache_planning_cases.json`` — outputs of the reference's cache-pool planner
  (runtime/cache_planning.py) on seeded routing traces and small inputs.
"""
from __future__ import annotations

import ast
import hashlib
import importlib.util
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.path.join(REPO, "zipmoe-icml26_b200"))

from oracle import codec  # noqa: E402
from zmoe import synthetic as syn  # noqa: E402


def digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        if isinstance(t, torch.Tensor):
            t = t.detach().contiguous().view(torch.uint8).numpy() if t.dtype != torch.uint8 else t.numpy()
        h.update(np.ascontiguousarray(t).tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------
# codec
# ---------------------------------------------------------------------------
def codec_cases():
    gen = torch.Generator().manual_seed(0)
    cases = {
        "normal_64x256": (torch.randn(64, 256, generator=gen) * 0.02).to(torch.bfloat16),
        "normal_ragged_37x53": (torch.randn(37, 53, generator=gen) * 0.08).to(torch.bfloat16),
        "zeros_32x512": torch.zeros(32, 512, dtype=torch.bfloat16),
        "const_16x1000": torch.full((16, 1000), 0.0123, dtype=torch.bfloat16),
        "tiny_1": torch.tensor([1.5], dtype=torch.bfloat16),
        "tiny_5": torch.tensor([1.0, -2.0, 3.0, 0.0, -0.5], dtype=torch.bfloat16),
        "random_bits_4099": torch.randint(0, 65536, (4099,), generator=gen, dtype=torch.int32)
        .to(torch.int16).view(torch.bfloat16),
        "normal_32x2048": (torch.randn(32, 2048, generator=gen) * 0.02).to(torch.bfloat16),
    }
    out = {}
    names = []
    for name, t in cases.items():
        bits = codec.bf16_bits(t)
        out[name + "__bits"] = bits
        for chunks in (1, 3, 5):
            if bits.size < chunks:
                continue
            for cod in ("LZ4HC", "LZ4"):
                key = f"{name}__c{chunks}__{cod}"
                blocks, osz, sm = codec.encode_tensor(bits, chunks, cod, 9, 5)
                exp_dec = np.concatenate([codec.lz4_decompress(b, o) for b, o in zip(blocks, osz)])
                assert np.array_equal(exp_dec, codec.split_planes(bits)[0])
                out[key + "__osz"] = np.array(osz, dtype=np.int64)
                out[key + "__csz"] = np.array([len(b) for b in blocks], dtype=np.int64)
                out[key + "__blocks"] = np.frombuffer(b"".join(blocks), dtype=np.uint8)
                names.append(key)
    out["names"] = np.array(names)
    out["tensors"] = np.array(list(cases))
    out["lz4_version"] = np.array(codec.lz4_version())
    np.savez_compressed(os.path.join(HERE, "codec_cases.npz"), **out)
    print("codec cases:", len(names))


# ---------------------------------------------------------------------------
# MoE blocks from the reference's Python
# ---------------------------------------------------------------------------
class _CPUExecutor:
    """Stand-in for ExpertExecutor.dispatch_local (experts/expert_executor.py:40-84)."""

    def __init__(self, block):
        self.block = block

    def dispatch_local(self, hidden_states, router_mask, layer_id):
        mask = router_mask.view(-1, router_mask.shape[-1])
        h = hidden_states.view(-1, hidden_states.shape[-1])
        res = []
        for e in range(mask.shape[-1]):
            tok = mask[:, e].bool()
            if int(tok.sum()) == 0:
                continue
            res.append((self.block.experts[e](h[tok]), layer_id, e, 1))
        return res


def _load_qwen(ref):
    spec = importlib.util.spec_from_file_location("ref_qwen_block", os.path.join(ref, "customized", "qwen.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _load_deepseek(ref):
    """Build MoEGate / DeepseekV2MLP from modeling_deepseek.py's class bodies
    (the module itself imports symbols newer transformers dropped) and load
    customized/deepseek.py against them."""
    src = open(os.path.join(ref, "models", "deepseek", "modeling_deepseek.py")).read()
    tree = ast.parse(src)
    keep = [n for n in tree.body if isinstance(n, ast.ClassDef) and n.name in ("MoEGate", "DeepseekV2MLP")]
    import math
    import torch.nn.functional as F
    from torch import nn
    from torch.nn import init
    from transformers.activations import ACT2FN
    ns = {"torch": torch, "nn": nn, "F": F, "math": math, "init": init, "ACT2FN": ACT2FN}
    exec(compile(ast.Module(body=keep, type_ignores=[]), "modeling_deepseek.py", "exec"), ns)
    models_pkg = types.ModuleType("models")
    ds_pkg = types.ModuleType("models.deepseek")
    ds_pkg.MoEGate = ns["MoEGate"]
    ds_pkg.DeepseekV2MLP = ns["DeepseekV2MLP"]
    models_pkg.deepseek = ds_pkg
    sys.modules["models"] = models_pkg
    sys.modules["models.deepseek"] = ds_pkg
    nv = types.ModuleType("nvtx")
    nv.annotate = lambda *a, **k: (lambda f: f)
    sys.modules.setdefault("nvtx", nv)
    ex_pkg = types.ModuleType("experts")
    ex_mod = types.ModuleType("experts.expert_executor")
    ex_mod.ExpertExecutor = object
    ex_pkg.expert_executor = ex_mod
    sys.modules["experts"] = ex_pkg
    sys.modules["experts.expert_executor"] = ex_mod
    spec = importlib.util.spec_from_file_location("ref_deepseek_block", os.path.join(ref, "customized", "deepseek.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


QWEN_SMALL = syn.LayerShape(hidden=256, num_experts=8, inter=64, topk=4, kind=0,
                            shared_inter=128, shared_gate=True)
DEEPSEEK_SMALL = syn.LayerShape(hidden=256, num_experts=8, inter=64, topk=3, kind=0,
                                shared_inter=128, shared_gate=False, scaling=1.0)


def small_inputs(s: syn.LayerShape, tokens: int):
    w = syn.expert_weights(s, 1, std=0.05, seed=10)[0]
    wr, sg = syn.router_weights(s, std=0.05, seed=12)
    sh = syn.shared_weights(s, std=0.05, seed=14)
    x = syn.activations(tokens, s.hidden, seed=11)
    return x, wr, sg, w, sh


def qwen_block(ref, tokens=24):
    from transformers import Qwen2MoeConfig
    mod = _load_qwen(ref)
    s = QWEN_SMALL
    cfg = Qwen2MoeConfig(hidden_size=s.hidden, num_experts=s.num_experts, num_experts_per_tok=s.topk,
                         moe_intermediate_size=s.inter, shared_expert_intermediate_size=s.shared_inter,
                         norm_topk_prob=False, hidden_act="silu")
    blk = mod.Qwen2MoEBlock(cfg).to(torch.bfloat16).eval()
    x, wr, sg, w, sh = small_inputs(s, tokens)
    with torch.no_grad():
        blk.gate.weight.copy_(wr)
        blk.shared_expert_gate.weight.copy_(sg)
        for e in range(s.num_experts):
            blk.experts[e].gate_proj.weight.copy_(w[e][0])
            blk.experts[e].up_proj.weight.copy_(w[e][1])
            blk.experts[e].down_proj.weight.copy_(w[e][2])
        blk.shared_expert.gate_proj.weight.copy_(sh[0])
        blk.shared_expert.up_proj.weight.copy_(sh[1])
        blk.shared_expert.down_proj.weight.copy_(sh[2])
        blk.expert_executor = _CPUExecutor(blk)
        blk.layer_id = 0
        y = blk(x.view(1, tokens, s.hidden)).view(tokens, s.hidden)
        logits = blk.gate(x)
        rw = torch.softmax(logits, dim=1, dtype=torch.float)
        tw, ti = torch.topk(rw, s.topk, dim=-1)
    np.savez_compressed(os.path.join(HERE, "qwen_block.npz"),
                        out=y.float().numpy(), topk_idx=ti.numpy().astype(np.int32),
                        topk_w=tw.numpy(), logits=logits.float().numpy(),
                        input_digest=np.array(digest(x, wr, sg, *w[0], *sh)), tokens=np.array(tokens))
    print("qwen block:", tuple(y.shape))


def qwen_block_c2(ref, tokens=64):
    """The reference's Qwen2MoEBlock at the full Qwen1.5-MoE-A2.7B layer shape
    (hidden 2048, 60 experts of intermediate 1408, top-4, shared expert 5632
    with its sigmoid gate), with the seeded synthetic weights of the benchmark
    (zmoe.synthetic: experts seed 0, router seed 2, shared seed 4) and 64
    tokens (seed 21).  The reference block has no router bias, so none is
    used here.  The output is stored as BF16 bit patterns."""
    from transformers import Qwen2MoeConfig
    mod = _load_qwen(ref)
    s = syn.QWEN
    cfg = Qwen2MoeConfig(hidden_size=s.hidden, num_experts=s.num_experts, num_experts_per_tok=s.topk,
                         moe_intermediate_size=s.inter, shared_expert_intermediate_size=s.shared_inter,
                         norm_topk_prob=False, hidden_act="silu")
    blk = mod.Qwen2MoEBlock(cfg).to(torch.bfloat16).eval()
    w = syn.expert_weights(s, 1)[0]
    wr, sg = syn.router_weights(s)
    sh = syn.shared_weights(s)
    x = syn.activations(tokens, s.hidden, seed=21)
    with torch.no_grad():
        blk.gate.weight.copy_(wr)
        blk.shared_expert_gate.weight.copy_(sg)
        for e in range(s.num_experts):
            blk.experts[e].gate_proj.weight.copy_(w[e][0])
            blk.experts[e].up_proj.weight.copy_(w[e][1])
            blk.experts[e].down_proj.weight.copy_(w[e][2])
        blk.shared_expert.gate_proj.weight.copy_(sh[0])
        blk.shared_expert.up_proj.weight.copy_(sh[1])
        blk.shared_expert.down_proj.weight.copy_(sh[2])
        blk.expert_executor = _CPUExecutor(blk)
        blk.layer_id = 0
        y = blk(x.view(1, tokens, s.hidden)).view(tokens, s.hidden)
        logits = blk.gate(x)
        rw = torch.softmax(logits, dim=1, dtype=torch.float)
        tw, ti = torch.topk(rw, s.topk, dim=-1)
    np.savez_compressed(os.path.join(HERE, "qwen_block_c2.npz"),
                        out_bits=y.contiguous().view(torch.int16).numpy(),
                        logits_bits=logits.contiguous().view(torch.int16).numpy(),
                        topk_idx=ti.numpy().astype(np.int32),
                        topk_w=tw.numpy(), input_digest=np.array(digest(x, wr, sg, *w[0], *w[-1], *sh)),
                        tokens=np.array(tokens))
    print("qwen block (C2 shape):", tuple(y.shape))


def deepseek_block(ref, tokens=24):
    mod = _load_deepseek(ref)
    s = DEEPSEEK_SMALL

    class Cfg:
        pass

    cfg = Cfg()
    cfg.model_type = "deepseek_v2"
    cfg.num_experts_per_tok = s.topk
    cfg.n_routed_experts = s.num_experts
    cfg.routed_scaling_factor = s.scaling
    cfg.scoring_func = "softmax"
    cfg.aux_loss_alpha = 0.0
    cfg.seq_aux = False
    cfg.topk_method = "greedy"
    cfg.n_group = 1
    cfg.topk_group = 1
    cfg.norm_topk_prob = False
    cfg.hidden_size = s.hidden
    cfg.intermediate_size = s.inter
    cfg.moe_intermediate_size = s.inter
    cfg.n_shared_experts = s.shared_inter // s.inter
    cfg.hidden_act = "silu"
    blk = mod.DeepseekMoEBlock(cfg).to(torch.bfloat16).eval()
    x, wr, _, w, sh = small_inputs(s, tokens)
    with torch.no_grad():
        blk.gate.weight.data = wr.clone()
        for e in range(s.num_experts):
            blk.experts[e].gate_proj.weight.copy_(w[e][0])
            blk.experts[e].up_proj.weight.copy_(w[e][1])
            blk.experts[e].down_proj.weight.copy_(w[e][2])
        blk.shared_experts.gate_proj.weight.copy_(sh[0])
        blk.shared_experts.up_proj.weight.copy_(sh[1])
        blk.shared_experts.down_proj.weight.copy_(sh[2])
        blk.expert_executor = _CPUExecutor(blk)
        blk.layer_id = 0
        y = blk(x.view(1, tokens, s.hidden)).view(tokens, s.hidden)
        ti, tw, _ = blk.gate(x.view(1, tokens, s.hidden))
    np.savez_compressed(os.path.join(HERE, "deepseek_block.npz"),
                        out=y.float().numpy(), topk_idx=ti.numpy().astype(np.int32), topk_w=tw.float().numpy(),
                        input_digest=np.array(digest(x, wr, *w[0], *sh)), tokens=np.array(tokens))
    print("deepseek block:", tuple(y.shape))


def predictor_cases(ref):
    """Replays seeded Zipf-skewed activations through the reference's own
    ExpertPredictor (experts/expert_predictor.py) and records its predictions."""
    import json
    spec = importlib.util.spec_from_file_location("ref_expert_predictor",
                                                  os.path.join(ref, "experts", "expert_predictor.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    rng = np.random.default_rng(31)
    cases = []
    for layers, E, k, topk, window in ((3, 16, 4, 4, 30), (26, 64, 6, 8, 26 * 6 * 10), (2, 8, 2, 20, 7)):
        pred = mod.ExpertPredictor(layers, topk, window_size=window)
        p = 1.0 / np.arange(1, E + 1) ** 1.2
        p /= p.sum()
        steps = []
        for step in range(120):
            layer = step % layers
            ids = [int(e) for e in rng.choice(E, size=k, replace=False, p=p)]
            pred.update(layer, ids)
            nl, got = pred.predict_next_layer(layer)
            steps.append({"layer": layer, "experts": ids, "next": nl, "predicted": [int(e) for e in got]})
        cases.append({"layers": layers, "topk": topk, "window": window, "steps": steps})
    with open(os.path.join(HERE, "predictor_cases.json"), "w") as f:
        json.dump(cases, f)
    print("predictor cases:", sum(len(c["steps"]) for c in cases))


def cache_planning_cases(ref):
    """Runs the reference's runtime/cache_planning.py functions (PlanCache and
    the pieces it is built from) on seeded synthetic routing traces and small
    hand-picked inputs, and records their outputs.  Its one GPU query (the
    device's total memory) is answered with a fixed size."""
    import json
    import tempfile
    spec = importlib.util.spec_from_file_location("ref_cache_planning", os.path.join(ref, "runtime", "cache_planning.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    real = torch.cuda.get_device_properties
    out = {"calculate_prob": [], "delay_simu": [], "scale_to_k": [], "coverage_to_weight": [], "plan": []}
    rng = np.random.default_rng(47)
    for n in (0, 1, 5, 17):
        p = [float(v) for v in rng.uniform(0.0, 1.0, n)]
        out["calculate_prob"].append({"probs": p, "out": [float(v) for v in mod.CalculateProb(p)]})
    for args in ((4, 0, 0, 0.5, 0.2, 0.7, 3, 3, 4), (4, 2, 1, 0.5, 0.2, 0.7, 3, 3, 4), (8, 3, 5, 1.3, 0.05, 0.82, 5, 2, 7),
                 (6, 6, 0, 0.4, 0.3, 0.6, 3, 3, 2)):
        out["delay_simu"].append({"args": list(args), "out": float(mod.DelaySimu(*args))})
    for probs, k in (([0.5, 0.2, 0.2, 0.1], 2), ([0.7, 0.1, 0.1, 0.05, 0.05], 3), ([0.0, 0.0], 1),
                     ([float(v) for v in sorted(rng.zipf(1.3, 24).astype(float), reverse=True)], 6)):
        out["scale_to_k"].append({"probs": probs, "k": k, "out": [float(v) for v in mod.scale_to_k(probs, k)]})
    for n, k in ((8, 2), (16, 4), (60, 4)):
        curve = 1.0 / np.arange(1, n + 1) ** 1.1
        target = mod.scale_to_k(list(curve / curve.sum()), k)
        out["coverage_to_weight"].append({"target": [float(v) for v in target], "k": k,
                                          "out": [float(v) for v in mod.CoverageToWeight(target, k)]})
    # PlanCache on seeded traces: trace[prompt][layer][expert] = invocations
    plans = ((24, 4, 16, 4, 4, 3, 1000, 432000, 0.5, 0.05), (40, 6, 16, 2, 8, 3, 1000, 600000, 0.5, 0.01),
             (30, 3, 20, 4, 5, 2, 2048, 2400000, 0.6, 0.05))
    for prompts, layers, E, k, batch, tensors, elems, total_memory, dev_ratio, step in plans:
        pop = 1.0 / np.arange(1, E + 1) ** 1.2
        pop /= pop.sum()
        trace = []
        for _ in range(prompts):
            per_layer = []
            for _ in range(layers):
                counts = np.zeros(E, dtype=np.int64)
                for _ in range(6):                                  # 6 tokens per prompt
                    counts[rng.choice(E, size=k, replace=False, p=rng.permutation(pop))] += 1
                per_layer.append([int(c) for c in counts])
            trace.append(per_layer)
        torch.cuda.get_device_properties = lambda i, m=total_memory: types.SimpleNamespace(total_memory=m)
        try:
            with tempfile.NamedTemporaryFile(suffix=".pt") as f:
                torch.save(trace, f.name)
                dist = mod.ObtainDistFromTrace(batch, f.name)
                args = dict(batch_size=batch, k=k, num_experts=E, num_sparse_layers=layers, tensors_per_expert=tensors,
                            num_elements_per_tensor=elems, compression_ratio=0.72, num_file_chunks=3,
                            compute_pool_size=4, device_memory_ratio=dev_ratio, decompression_delay=0.45,
                            SM_IO_delay=0.21, step_size=step)
                ratio, feasible = mod.PlanCache(trace_path=f.name, **args)
        finally:
            torch.cuda.get_device_properties = real
        out["plan"].append({"trace": trace, "total_memory": total_memory, "args": args, "dist": [float(v) for v in dist],
                            "ratio": float(ratio), "feasible": bool(feasible)})
    with open(os.path.join(HERE, "cache_planning_cases.json"), "w") as f:
        json.dump(out, f)
    print("cache planning cases:", {kk: len(v) for kk, v in out.items()},
          [(c["ratio"], c["feasible"]) for c in out["plan"]])


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <path of the reference checkout>")
    ref = sys.argv[1]
    only = sys.argv[2:]
    if only:
        for name in only:
            globals()[name](ref) if name != "codec_cases" else codec_cases()
        sys.exit(0)
    codec_cases()
    qwen_block(ref)
    qwen_block_c2(ref)
    deepseek_block(ref)
    predictor_cases(ref)
    cache_planning_cases(ref)
