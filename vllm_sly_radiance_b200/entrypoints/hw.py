"""Hardware detection and KV-cache calibration for the launcher.

* ``detect_gpus``: the CUDA devices this host can serve on (NVML, read-only queries), with a
  memory floor that drops small display adapters, and the tensor-parallel size: the largest
  allowed degree that fits the device count and divides the model's head counts (q heads, GDN
  key and value heads; kv heads may be replicated when TP exceeds them).
* ``calibrate_kv``: the number of KV blocks that survives a chunk-sized prefill plus a short
  decode, found by search (grow while it survives, then bisect), written to a local profile
  table that the engine reads when no explicit ``num_kv_blocks`` is given.

Reference behaviour: gpu-detect.sh (sysfs enumeration, VRAM floor, TP must divide 24 / 16 / 48,
profile lookup) and calibrate-kv.sh (raise the pin until startup + one CHUNK prefill + decode
stops surviving, back off, save to ~/.cache/.../kv-profiles.local.tsv).  Nothing here changes a
device setting."""
from __future__ import annotations

import csv
import os
from dataclasses import dataclass
from typing import Callable, Optional

PROFILE_PATH = os.path.join(os.path.expanduser("~"), ".cache", "radiance-b200", "kv-profiles.tsv")
TP_ALLOWED = (8, 4, 2, 1)


@dataclass
class GpuInfo:
    index: int
    name: str
    mem_mib: int


def nvml_gpus() -> list[GpuInfo]:
    """Devices from NVML (name, total memory); [] when NVML is unavailable."""
    try:
        import pynvml
        pynvml.nvmlInit()
    except Exception:
        return []
    try:
        out = []
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            name = pynvml.nvmlDeviceGetName(h)
            name = name.decode() if isinstance(name, bytes) else name
            out.append(GpuInfo(i, name, pynvml.nvmlDeviceGetMemoryInfo(h).total // (1 << 20)))
        return out
    finally:
        pynvml.nvmlShutdown()


def pick_tp(num_gpus: int, mcfg, allowed=TP_ALLOWED) -> int:
    """Largest allowed TP degree <= num_gpus that divides the q heads and the GDN key / value
    heads (kv heads are replicated when TP exceeds them, so TP must be a multiple of them or
    divide them)."""
    for tp in sorted(allowed, reverse=True):
        if tp > num_gpus:
            continue
        if mcfg.num_q_heads % tp or mcfg.gdn_num_k_heads % tp or mcfg.gdn_num_v_heads % tp:
            continue
        if mcfg.num_kv_heads % tp and tp % mcfg.num_kv_heads:
            continue
        return tp
    return 1


def detect_gpus(mcfg, gpus: Optional[list[GpuInfo]] = None, min_mib: int = 8192,
                allowed=TP_ALLOWED) -> dict:
    gpus = nvml_gpus() if gpus is None else gpus
    usable = [g for g in gpus if g.mem_mib >= min_mib]
    skipped = [g for g in gpus if g.mem_mib < min_mib]
    tp = pick_tp(len(usable), mcfg, allowed) if usable else 0
    sig = usable[0].name if usable else None
    return {"gpus": [vars(g) for g in usable], "skipped": [vars(g) for g in skipped],
            "tensor_parallel_size": tp, "signature": sig,
            "kv_blocks_pin": lookup_pin(sig, mcfg.name, tp) if sig else None}


# ---- KV calibration ----------------------------------------------------------------------
def _key(sig, model, tp, max_num_seqs=None, chunk=None):
    return (str(sig), str(model), str(tp), str(max_num_seqs or ""), str(chunk or ""))


def lookup_pin(sig, model, tp, max_num_seqs=None, chunk=None, path: str = PROFILE_PATH):
    """num_kv_blocks measured for (device, model, TP[, batch shape]); None when absent."""
    if not os.path.exists(path):
        return None
    best = None
    with open(path) as f:
        for row in csv.reader(f, delimiter="\t"):
            if len(row) != 6 or row[0].startswith("#"):
                continue
            if tuple(row[:3]) != _key(sig, model, tp)[:3]:
                continue
            if (max_num_seqs and row[3] and row[3] != str(max_num_seqs)) or \
                    (chunk and row[4] and row[4] != str(chunk)):
                continue
            best = int(row[5])
    return best


def save_pin(sig, model, tp, max_num_seqs, chunk, blocks: int, path: str = PROFILE_PATH):
    os.makedirs(os.path.dirname(path), exist_ok=True)
    rows = []
    if os.path.exists(path):
        with open(path) as f:
            rows = [r for r in csv.reader(f, delimiter="\t")
                    if len(r) == 6 and tuple(r[:5]) != _key(sig, model, tp, max_num_seqs, chunk)]
    rows.append(list(_key(sig, model, tp, max_num_seqs, chunk)) + [str(blocks)])
    with open(path, "w", newline="") as f:
        w = csv.writer(f, delimiter="\t")
        w.writerow(["# device", "model", "tp", "max_num_seqs", "chunk", "num_kv_blocks"])
        w.writerows(rows)


def search_blocks(survives: Callable[[int], bool], start: int, step: float = 1.25,
                  tol: int = 16, max_tries: int = 24) -> int:
    """Largest block count n (within tol) with survives(n): grow geometrically from a start that
    survives, then bisect between the last survivor and the first failure."""
    if not survives(start):
        lo, hi = 0, start
    else:
        lo, hi, tries = start, None, 0
        while hi is None and tries < max_tries:
            nxt = int(lo * step) + tol
            if survives(nxt):
                lo = nxt
            else:
                hi = nxt
            tries += 1
        if hi is None:
            return lo
    while hi - lo > tol:
        mid = (lo + hi) // 2
        if survives(mid):
            lo = mid
        else:
            hi = mid
    return lo


def engine_survives(cfg, blocks: int) -> bool:
    """Build the engine with `blocks` KV blocks, run one chunk-sized prefill and a short decode;
    False on a CUDA out-of-memory error (the engine is released either way)."""
    import gc

    import torch

    from ..engine.llm_engine import LLMEngine
    from ..engine.request import SamplingParams
    import dataclasses
    eng = None
    try:
        eng = LLMEngine(dataclasses.replace(cfg, num_kv_blocks=blocks))
        n = min(cfg.max_num_batched_tokens, cfg.max_model_len - 16)
        eng.generate([list(range(3, 3 + n))], SamplingParams(temperature=0, max_tokens=4,
                                                             ignore_eos=True))
        return True
    except torch.cuda.OutOfMemoryError:
        return False
    finally:
        del eng
        gc.collect()
        torch.cuda.empty_cache()


def calibrate_kv(cfg, survives: Optional[Callable[[int], bool]] = None, sig: Optional[str] = None,
                 path: str = PROFILE_PATH, save: bool = True) -> int:
    import torch
    if survives is None:
        survives = lambda n: engine_survives(cfg, n)        # noqa: E731
    if sig is None:
        sig = torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu"
    # start from the engine's own sizing (what a profile run would pick)
    start = max(64, cfg.num_kv_blocks or 1024)
    blocks = search_blocks(survives, start)
    if save:
        save_pin(sig, cfg.model, cfg.tensor_parallel_size, cfg.max_num_seqs,
                 cfg.max_num_batched_tokens, blocks, path)
    return blocks
