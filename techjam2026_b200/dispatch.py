"""Frozen dispatch table keyed on (arch, I/O dtype, shape signature).

Mirrors the reference's `DispatchTable.load_for(spec).lookup(arch, dtype, cfg,
smem_kb) -> (Plan, source)` (kernelforge/dispatch.py:247-288) with the same
fallback order -- exact entry, then a conservative plan when the table knows
the arch but not the shape ("nearest"), then the built-in default -- but the
table is for sm_100 only and a Plan describes the sm_100a CUDA path:
tile choices for the four GEMMs and the numerics switches, all of them
covered by the parity tests. Entries live in dispatch_sm_100.json next to
this file.
"""
from __future__ import annotations

import dataclasses
import json
import math
import os
from typing import Dict, List, Optional, Tuple

import torch

from .configs import signature

TABLE_DIR = os.path.dirname(os.path.abspath(__file__))
SUPPORTED_ARCHES = ("sm_100", "sm_100a")


@dataclasses.dataclass(frozen=True)
class Plan:
    name: str = "bf16x3-gemm+tf32-attn+graph"
    # Capture the whole multi-layer forward in one CUDA graph.
    cuda_graph: bool = True
    # Precision of each GEMM: "tf32" (one TF32 pass), "3xtf32" (fp32
    # operands, split in shared memory) or "bf16x3" (operands kept as bf16
    # hi/lo planes by their producers; three BF16 MMAs per k step), the last
    # two error-compensated (hi*hi + hi*lo + lo*hi). Plain TF32 everywhere
    # fails the organiser's gate against the fp32 reference on the 6-layer
    # config (envelope 1.2-1.4); compensated GEMMs with TF32 attention
    # measure 0.41-0.63 on every config. bf16x3 needs half the MMA time and a
    # quarter of the shared-memory operand traffic of 3xtf32 per k element.
    prec_qkv: str = "bf16x3"
    prec_out: str = "bf16x3"
    prec_ffn1: str = "bf16x3"
    prec_ffn2: str = "bf16x3"
    # Round operands that feed a plain TF32 MMA (attention, and any GEMM not
    # split) to the nearest TF32 value where they are produced, so the tensor
    # core's truncation of the low mantissa bits is a no-op: unbiased operand
    # error instead of round-toward-zero.
    round_tf32: bool = True
    # Attention writes 0 for query tiles without a valid token instead of
    # computing them (those rows are masked right after out_proj).
    skip_empty_queries: bool = True
    # GEMMs compute only 128-row tiles holding a real token and the non-final
    # norms leave padded rows untouched (every consumer masks those rows).
    skip_padded_rows: bool = True
    # N tile of each GEMM (0 = pick by wave quantisation at launch).
    bn_qkv: int = 0
    bn_out: int = 0
    bn_ffn1: int = 0
    bn_ffn2: int = 0
    # bf16x3 GEMM on CTA pairs (tcgen05 cta_group::2, 256 x bn tiles, bn 128
    # or 256): each SM stages half of B, which relieves shared-memory
    # bandwidth on large GEMMs (c3b/c4: 9-18% faster per GEMM at bn 256);
    # on small ones (c2) the coarser tiles lose. Bit-identical output.
    pair_qkv: bool = False
    pair_out: bool = False
    pair_ffn1: bool = False
    pair_ffn2: bool = False
    # Stream-K scheduling of a bf16x3 GEMM (kf_gemm_bf16x3_sk): every SM takes
    # an even share of the (tile, k block) pairs, for GEMMs whose tiles fill
    # only part of one wave (c2's N = 512 GEMMs: 108 tiles on 148 SMs). Split
    # tiles are summed in a fixed order: deterministic, not bit-identical.
    sk_qkv: bool = False
    sk_out: bool = False
    sk_ffn1: bool = False
    sk_ffn2: bool = False

    # Attention walks the batch rows longest first (kf_batch_order, one small
    # kernel per forward): a launch of several waves then ends on short
    # rows instead of a late long row's heavy causal tiles. Schedule only;
    # bit-identical output.
    order_rows: bool = False

    # FFN1 and FFN2 run over the valid tokens only, packed into consecutive
    # rows (kf_pack_rows builds the row map once per forward): LN2 writes its
    # output at a token's packed row, the norm after FFN2 reads FFN2's output
    # from there (kf_ln_add_mask_rows). The padded rows inside a sequence's
    # last 128-row tile are not computed (c4: 6 % of the GEMM rows, c2 14 %).
    # Every row's arithmetic is unchanged: bit-identical output.
    packed_ffn: bool = True

    # Persistent attention over a work list built once per forward
    # (kf_attn_schedule + kf_flash_fwd_tf32_sched): one CTA per resident
    # slot takes (row, head, query tile) items longest row first, heaviest
    # causal tile first, keeping its barriers, TMEM and pipelines between
    # items; query tiles without a valid query are not touched at all (their
    # rows are padding, which every consumer masks). Bit-identical rows for
    # every valid query.
    attn_persistent: bool = True

    # Narrow I/O dtypes (float16/bfloat16): run the organiser's own layer,
    # captured whole into one CUDA graph, instead of these kernels. At those
    # dtypes the gate only admits the reference's exact arithmetic
    # (techjam2026_b200/exact.py); never set for float32.
    exact_reference: bool = False

    def gemm_precisions(self) -> dict:
        return {"qkv": self.prec_qkv, "out": self.prec_out, "ffn1": self.prec_ffn1,
                "ffn2": self.prec_ffn2}

    def describe(self) -> str:
        precs = self.gemm_precisions()
        if len(set(precs.values())) == 1:
            bits = [f"{self.prec_qkv}-gemm"]
        else:
            bits = ["gemm[" + ",".join(f"{k}={v}" for k, v in precs.items()) + "]"]
        bits.append("tf32-attn")
        if self.round_tf32:
            bits.append("rna-operands")
        if self.skip_empty_queries:
            bits.append("skip-empty-q")
        if self.skip_padded_rows:
            bits.append("skip-padded-rows")
        if self.packed_ffn:
            bits.append("packed-ffn")
        if self.attn_persistent:
            bits.append("persistent-attn")
        elif self.order_rows:
            bits.append("rows-longest-first")
        if self.exact_reference:
            return "exact-reference+cuda-graph"
        if self.cuda_graph:
            bits.append("cuda-graph")
        tiles = (self.bn_qkv, self.bn_out, self.bn_ffn1, self.bn_ffn2)
        if any(tiles):
            bits.append("bn=" + "/".join(str(t or "auto") for t in tiles))
        pairs = (self.pair_qkv, self.pair_out, self.pair_ffn1, self.pair_ffn2)
        if any(pairs):
            bits.append("cta-pair=" + "/".join("y" if p else "n" for p in pairs))
        sks = (self.sk_qkv, self.sk_out, self.sk_ffn1, self.sk_ffn2)
        if any(sks):
            bits.append("stream-k=" + "/".join("y" if p else "n" for p in sks))
        return " ".join(bits)


DEFAULT_PLAN = Plan()
# float16 / bfloat16 I/O: the reference's own forward in one CUDA graph.
EXACT_PLAN = Plan(name="exact-reference+graph", exact_reference=True)
# For shapes never measured: same arithmetic, automatic tiles.
CONSERVATIVE_PLAN = dataclasses.replace(DEFAULT_PLAN, name=DEFAULT_PLAN.name + "(auto-tiles)")


@dataclasses.dataclass
class Entry:
    signature: str
    dtype: str
    arch: str
    plan: Plan
    note: str = ""

    def to_json(self) -> dict:
        d = dataclasses.asdict(self)
        d["plan"] = dataclasses.asdict(self.plan)
        return d

    @staticmethod
    def from_json(d: dict) -> "Entry":
        return Entry(d["signature"], d["dtype"], d["arch"], Plan(**d["plan"]), d.get("note", ""))


def _norm_arch(arch: str) -> str:
    return "sm_100" if arch in SUPPORTED_ARCHES else arch


class DispatchTable:
    def __init__(self, entries: Optional[List[Entry]] = None):
        self.entries: List[Entry] = list(entries or [])
        self._index: Dict[Tuple[str, str, str], Entry] = {
            (_norm_arch(e.arch), e.dtype, e.signature): e for e in self.entries}

    @staticmethod
    def path_for(arch: str) -> str:
        return os.path.join(TABLE_DIR, f"dispatch_{_norm_arch(arch)}.json")

    @staticmethod
    def load(arch: str = "sm_100") -> "DispatchTable":
        path = DispatchTable.path_for(arch)
        if not os.path.exists(path):
            return DispatchTable([])
        with open(path, encoding="utf-8") as f:
            blob = json.load(f)
        return DispatchTable([Entry.from_json(e) for e in blob.get("entries", [])])

    @staticmethod
    def load_for(spec) -> "DispatchTable":
        return DispatchTable.load(spec.arch)

    def save(self, arch: str = "sm_100") -> str:
        path = self.path_for(arch)
        with open(path, "w", encoding="utf-8") as f:
            json.dump({"arch": _norm_arch(arch),
                       "entries": [e.to_json() for e in self.entries]}, f, indent=2)
            f.write("\n")
        return path

    def lookup(self, arch: str, dtype: torch.dtype, cfg, smem_kb: float = 227.0
               ) -> Tuple[Plan, str]:
        a = _norm_arch(arch)
        if a != "sm_100":
            raise RuntimeError(f"no kernels for {arch}: this build targets sm_100a only")
        dt = str(dtype).replace("torch.", "")
        if dt in ("float16", "bfloat16"):
            # The gate admits only the reference's exact arithmetic there
            # (the reference's own table ships exact plans for these dtypes).
            return EXACT_PLAN, "exact-dtype"
        if dt != "float32":
            raise RuntimeError(f"I/O dtype {dt} is not implemented")
        sig = signature(cfg)
        hit = self._index.get((a, dt, sig))
        if hit is not None:
            return hit.plan, "exact"
        same_arch = [e for e in self.entries if _norm_arch(e.arch) == a and e.dtype == dt]
        if same_arch:
            # Nearest: the same layer shape at another batch size (a batch
            # slice, or one rank's shard of a multi-GPU batch) keeps the
            # measured plan of the closest batch; any other shape gets the
            # same arithmetic with tiles chosen at launch.
            rest = sig.split("-", 1)[1]
            same_layer = [e for e in same_arch if e.signature.split("-", 1)[1] == rest]
            if same_layer:
                B = max(1, cfg.batch_size)
                best = min(same_layer,
                           key=lambda e: abs(math.log(max(1, int(e.signature.split("-", 1)[0][1:]))) -
                                             math.log(B)))
                return best.plan, "nearest"
            return CONSERVATIVE_PLAN, "nearest"
        return DEFAULT_PLAN, "default"


@dataclasses.dataclass(frozen=True)
class GPUSpec:
    name: str
    arch: str
    sm_count: int
    shared_mem_per_block_kb: float
    total_mem_gb: float


def probe(device: Optional[int] = None) -> GPUSpec:
    """The current CUDA device, described for dispatch."""
    dev = torch.cuda.current_device() if device is None else device
    p = torch.cuda.get_device_properties(dev)
    smem = getattr(p, "shared_memory_per_block_optin", 232448) / 1024.0
    return GPUSpec(p.name, f"sm_{p.major}{p.minor}", p.multi_processor_count, smem,
                   p.total_memory / 1e9)
