"""Shared test plumbing: golden fixtures, oracle runs and device runs of a
:class:`casegen.Case`."""
from __future__ import annotations

from pathlib import Path

import numpy as np

from casegen import Case, golden_cases

GOLDEN = Path(__file__).resolve().parent / "golden"

# Tolerances (max-abs on attention outputs, whose entries are O(1)).
TOL_FP32 = 2e-5       # kernel (fp32) vs reference CPU path
TOL_TF32 = 1e-3       # kernel with tcgen05 TF32 prefill tiles vs reference
TOL_ORACLE = 5e-6     # C restatement vs the reference's own build (-ffast-math)


# LM-head logits (device model vs the reference's), relative to the row's
# largest |logit|: fp32 GEMMs in a different summation order than the
# reference's k-outer loop
LOGIT_RTOL = 1e-5


def load_trace(name: str):
    """A reference token trace: (model config, the npz, parsed steps)."""
    from oracle.oracle import read_trace
    z = np.load(GOLDEN / f"{name}.npz")
    v, d, layers, heads, hd, ffn = (int(x) for x in z["model"])
    cfg = dict(vocab=v, hidden=d, layers=layers, heads=heads, head_dim=hd, ffn=ffn)
    return cfg, z, read_trace(z["trace"])


def trace_requests(z):
    """(prompts, max_new) of a token trace; sequence i + 1 is request i."""
    lens, toks = z["prompt_lens"], z["prompt_tokens"]
    offs = np.concatenate([[0], np.cumsum(lens)])
    return [toks[offs[i]:offs[i + 1]] for i in range(len(lens))], [int(x) for x in z["max_new"]]


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def golden_names() -> list[str]:
    return [c.name for c in golden_cases()]


def golden_case(name: str) -> Case:
    for c in golden_cases():
        if c.name == name:
            return c
    raise KeyError(name)


def layout_of(case: Case, KVLayout):
    return KVLayout(case.num_blocks, case.num_layers, case.block_size, case.num_heads,
                    case.head_dim)


def metadata(oracle, case: Case) -> dict:
    """Flatten + slot mapping of the new tokens, and of the cached history."""
    fl = oracle.flatten(case.num_computed, case.total_len)
    slots = oracle.slot_mapping(fl["cu_seqlens_q"], fl["context_lens"], case.block_tables,
                                case.block_size)
    hist_cu = np.concatenate([[0], np.cumsum(case.num_computed)]).astype(np.int32)
    hist_slots = oracle.slot_mapping(hist_cu, case.num_computed, case.block_tables,
                                     case.block_size)
    return dict(cu_seqlens_q=fl["cu_seqlens_q"], context_lens=fl["context_lens"], slots=slots,
                hist_slots=hist_slots, positions=fl["positions"])


def oracle_run(oracle, case: Case, use_f64: bool = False):
    """Host arenas written by the oracle and the oracle attention, per layer."""
    from oracle.oracle import KVLayout
    lay = layout_of(case, KVLayout)
    md = metadata(oracle, case)
    ka = np.zeros(lay_shape(case), np.float32)
    va = np.zeros_like(ka)
    out = np.zeros((case.num_layers, case.n_tokens, case.hidden), np.float32)
    for layer in range(case.num_layers):
        oracle.reshape_and_cache(case.hist_k[layer], case.hist_v[layer], ka, va, md["hist_slots"],
                                 layer, lay)
        oracle.reshape_and_cache(case.k[layer], case.v[layer], ka, va, md["slots"], layer, lay)
        out[layer] = oracle.paged_attention(case.q[layer], ka, va, case.block_tables,
                                            md["cu_seqlens_q"], md["context_lens"], layer,
                                            case.scale, lay, use_f64=use_f64)
    return ka, va, out, md


def lay_shape(case: Case):
    return (case.num_blocks, case.num_layers, case.block_size, case.hidden)


def device_run(nv, oracle, case: Case, precision: int = 0, workspace_pad: int = 0):
    """Runs the case through the C ABI on cuda:0: history and new tokens written
    by nvllm_reshape_and_cache, then nvllm_paged_attention per layer."""
    import torch
    lay = layout_of(case, nv.KVLayout)
    md = metadata(oracle, case)
    dev = torch.device("cuda:0")
    ka = torch.zeros(lay_shape(case), dtype=torch.float32, device=dev)
    va = torch.zeros_like(ka)
    bt = torch.from_numpy(case.block_tables).to(dev)
    cu = torch.from_numpy(md["cu_seqlens_q"]).to(dev)
    ctx = torch.from_numpy(md["context_lens"]).to(dev)
    slots = torch.from_numpy(md["slots"]).to(dev)
    hslots = torch.from_numpy(md["hist_slots"]).to(dev)
    max_q = int(case.q_lens.max())
    max_ctx = int(case.total_len.max())
    ws = nv.alloc_workspace(len(case.total_len), max_q, max_ctx, lay, device=dev)
    if workspace_pad:
        ws = torch.empty(ws.numel() + workspace_pad, dtype=torch.uint8, device=dev)
    outs = []
    for layer in range(case.num_layers):
        if len(md["hist_slots"]):
            nv.reshape_and_cache(torch.from_numpy(case.hist_k[layer]).to(dev),
                                 torch.from_numpy(case.hist_v[layer]).to(dev), ka, va, hslots,
                                 layer, lay)
        nv.reshape_and_cache(torch.from_numpy(case.k[layer]).to(dev),
                             torch.from_numpy(case.v[layer]).to(dev), ka, va, slots, layer, lay)
        q = torch.from_numpy(case.q[layer]).to(dev)
        out = torch.full_like(q, float("nan"))
        nv.paged_attention(out, q, ka, va, bt, cu, ctx, max_q, max_ctx, layer, lay,
                           scale=case.scale, precision=precision, workspace=ws)
        outs.append(out)
    torch.cuda.synchronize()
    status = nv.get_last_error()
    return (ka.cpu().numpy(), va.cpu().numpy(), torch.stack(outs).cpu().numpy(), status)
