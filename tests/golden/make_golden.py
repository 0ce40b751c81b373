"""Generate the golden fixtures by running the REFERENCE implementation.

Run from the repository root with ``FLASHDEC_REF`` naming a checkout of
cysong2025/flashdec (or a directory the reference is installed into, such as
``baseline/_ref``):

    FLASHDEC_REF=<path to the reference> python tests/golden/make_golden.py

It imports the reference's own oracles -- ``flashdec.paged_reference``,
``flashdec.rope``, ``flashdec.cache.PagedKVCache`` and
``flashdec.vllm_backend._select_num_splits`` -- feeds them the seeded inputs
of ``tests/golden/cases.py`` on the CPU, and writes:

* ``attn_golden.npz``   -- reference paged-decode outputs per attention case
  (and per fused-append case: the reference oracle run on the cache after the
  current token was appended, exactly as the reference's own fused-append
  tests build their expectation);
* ``rope_golden.npz``   -- reference ``apply_rope`` of q and k per RoPE case,
  plus the reference's fp32 ``inv_freq`` tables;
* ``ledger_golden.json`` -- a trace of block tables / slots / lengths produced
  by the reference ``PagedKVCache`` for a scripted request lifecycle;
* ``split_policy_golden.json`` -- ``_select_num_splits`` over a grid.

The fixtures are small (a few hundred KB) and are committed; the tests never
need the reference at run time.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

from tests.golden import cases  # noqa: E402

TORCH_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _t(a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(TORCH_DTYPES[dtype])


def _bits(t):
    """float32 payload for fp32 tensors, uint16 bit patterns for 16-bit ones."""
    if t.dtype == torch.float32:
        return t.numpy().astype(np.float32)
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def attention_fixtures():
    from flashdec.paged_reference import paged_decode_attention_ref

    out = {}
    for name in cases.ATTN_CASES:
        c = cases.make_attn_case(name)
        res = paged_decode_attention_ref(
            _t(c["q"], c["dtype"]),
            _t(c["k_cache"], c["dtype"]),
            _t(c["v_cache"], c["dtype"]),
            torch.from_numpy(c["block_tables"]),
            torch.from_numpy(c["seq_lens"]),
            sm_scale=c["sm_scale"],
            kv_layout=c["kv_layout"],
        )
        out[f"{name}/out"] = _bits(res)
        out[f"{name}/digest"] = np.array(_digest(c["q"], c["k_cache"], c["v_cache"], c["block_tables"]))
    for name in cases.APPEND_ATTN_CASES:
        c = cases.make_append_attn_case(name)
        k = _t(c["k_cache"], c["dtype"])
        v = _t(c["v_cache"], c["dtype"])
        bs = c["block_size"]
        for row, slot in enumerate(c["slot_mapping"].tolist()):
            k[slot // bs, :, slot % bs, :] = _t(c["append_k"][row], c["dtype"])
            v[slot // bs, :, slot % bs, :] = _t(c["append_v"][row], c["dtype"])
        res = paged_decode_attention_ref(
            _t(c["q"], c["dtype"]), k, v,
            torch.from_numpy(c["block_tables"]), torch.from_numpy(c["seq_lens"]),
        )
        out[f"{name}/out"] = _bits(res)
        out[f"{name}/digest"] = np.array(_digest(c["q"], c["k_cache"], c["append_k"], c["block_tables"]))
    return out


def rope_fixtures():
    from flashdec.rope import apply_rope

    out = {}
    for name in cases.ROPE_CASES:
        c = cases.make_rope_case(name)
        pos = torch.from_numpy(c["positions"])
        q = apply_rope(_t(c["q"], c["dtype"]), pos, rotary_dim=c["rotary_dim"], base=c["base"])
        k = apply_rope(_t(c["k"], c["dtype"]), pos, rotary_dim=c["rotary_dim"], base=c["base"])
        out[f"{name}/q_rot"] = _bits(q)
        out[f"{name}/k_rot"] = _bits(k)
        out[f"{name}/digest"] = np.array(_digest(c["q"], c["k"], c["positions"]))
    for rd, base in [(128, 1e6), (128, 1e4), (4, 1e4), (32, 1e4), (64, 5e5)]:
        steps = torch.arange(0, rd, 2, dtype=torch.float32)
        out[f"inv_freq/{rd}/{base:g}"] = torch.pow(base, -steps / rd).numpy()
    # reference tests/test_rope_append.py:73-95 known answer, produced by the reference
    x = torch.tensor([[[1.0, 2.0, 3.0, 4.0]], [[1.0, 2.0, 3.0, 4.0]]])
    out["known_answer/out"] = apply_rope(x, torch.tensor([0, 1])).numpy()
    return out


def ledger_fixture():
    """Scripted PagedKVCache lifecycle; records every observable integer."""
    from flashdec.cache import PagedKVCache

    cache = PagedKVCache(num_layers=2, num_kv_heads=1, head_dim=2, block_size=8,
                         max_blocks=24, dtype=torch.float32, device="cpu",
                         prefix_cache_capacity_blocks=6)
    log = []

    def active():
        return [rid for rid, st in cache._requests.items() if st.status == "active"]

    def snap(tag, extra=None):
        ids = active()
        rec = {
            "tag": tag,
            "free": list(cache._free_blocks),
            "state_version": cache.state_version,
            "block_ids": {str(r): list(cache.request_state(r)["block_ids"]) for r in ids},
            "seq_lens": {str(r): cache.request_state(r)["seq_len"] for r in ids},
        }
        if ids:
            rec["active"] = [str(r) for r in ids]
            rec["block_tables"] = cache.block_tables(ids).tolist()
        m = cache.metrics()
        rec["metrics"] = {k: m[k] for k in LEDGER_METRICS}
        if extra:
            rec.update(extra)
        log.append(rec)

    def kv(n, val):
        return torch.full((n, 1, 2), float(val))

    prefix_k = torch.arange(2 * 2 * 1 * 8 * 2, dtype=torch.float32).reshape(2, 2, 1, 8, 2)
    cache.register_prefix("sys", prefix_k, prefix_k + 1000)
    snap("register_prefix")
    for rid in ("a", "b", "c"):
        cache.add_request(rid)
    cache.attach_prefix("c", "sys")
    snap("add_requests")
    for step in range(30):
        ids = active()
        if step % 3 == 1:
            ids = list(reversed(ids))
        tx = cache.begin_token(ids)
        extra = {
            "ids": [str(r) for r in ids],
            "positions": tx.positions.tolist(),
            "physical_block_ids": tx.physical_block_ids.tolist(),
            "block_offsets": tx.block_offsets.tolist(),
            "effective_seq_lens": tx.effective_seq_lens.tolist(),
            "tx_block_tables": tx.block_tables.tolist(),
        }
        for layer in range(2):
            cache.write_token_layer(tx, layer, kv(len(ids), step), kv(len(ids), -step))
        if step in (4, 11, 20):
            cache.abort_token(tx)
            snap(f"abort_{step}", extra)
        else:
            cache.commit_token(tx)
            snap(f"commit_{step}", extra)
        if step == 6:
            cache.finish_request("b")
            cache.add_request("d")
            snap("finish_b_add_d")
        if step == 12:
            cache.cancel_request("a")
            cache.add_request("e")
            cache.attach_prefix("e", "sys")
            cache.add_request("f")
            snap("cancel_a_add_e_f")
        if step == 24:
            cache.finish_request(active()[0])
            snap("finish_first")
    try:
        cache.evict_prefix("sys")
    except RuntimeError as exc:
        log.append({"tag": "evict_refused", "error": str(exc)})
    for rid in active():
        cache.finish_request(rid)
    snap("finish_all")
    released = cache.evict_prefix("sys")
    snap("evict_prefix", {"released": list(released)})
    small = PagedKVCache(num_layers=1, num_kv_heads=1, head_dim=2, block_size=2,
                         max_blocks=3, dtype=torch.float32, device="cpu")
    for rid in (1, 2, 3, 4):
        small.add_request(rid)
    err = None
    try:
        small.begin_token([1, 2, 3, 4])
    except RuntimeError as exc:
        err = str(exc)
    log.append({"tag": "capacity_failure", "error": err, "free": list(small._free_blocks),
                "capacity_failure_count": small.metrics()["capacity_failure_count"]})
    return log


LEDGER_METRICS = (
    "used_blocks", "free_blocks", "allocation_count", "fresh_allocation_count",
    "free_count", "reuse_count", "capacity_failure_count", "transaction_begin_count",
    "transaction_commit_count", "transaction_abort_count",
    "transaction_rollback_block_count", "resident_prefix_blocks", "prefix_hit_count",
    "prefix_eviction_count", "internal_fragmentation_tokens", "active_tokens",
    "physical_data_tokens", "reserved_tokens", "saved_prefix_blocks",
    "shared_prefix_blocks", "active_prefix_references",
)


def split_policy_fixture():
    from flashdec.vllm_backend import _select_num_splits

    rows = []
    for requested in (0, 1, 2, 4, 8, 16):
        for num_reqs in (1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 16, 32, 64, 128, 256):
            for hkv in (1, 2, 4, 8):
                for logical_blocks in (1, 2, 3, 4, 7, 8, 15, 16, 17, 32, 64, 128):
                    rows.append([requested, num_reqs, hkv, logical_blocks,
                                 _select_num_splits(requested, num_reqs=num_reqs,
                                                    num_kv_heads=hkv,
                                                    logical_blocks=logical_blocks)])
    return rows


def main():
    # the reference is imported lazily by each fixture function; importing
    # this module (for LEDGER_METRICS) needs no reference
    if not os.environ.get("FLASHDEC_REF"):
        sys.exit("set FLASHDEC_REF to a checkout (or install) of the reference, cysong2025/flashdec")
    sys.path.insert(0, os.environ["FLASHDEC_REF"])
    np.savez_compressed(HERE / "attn_golden.npz", **attention_fixtures())
    np.savez_compressed(HERE / "rope_golden.npz", **rope_fixtures())
    (HERE / "ledger_golden.json").write_text(json.dumps(ledger_fixture(), indent=0))
    try:
        rows = split_policy_fixture()
    except Exception as exc:  # vLLM / triton missing in this checkout's env
        print("split policy fixture skipped:", exc)
    else:
        (HERE / "split_policy_golden.json").write_text(json.dumps(rows))
    for p in sorted(HERE.glob("*_golden.*")):
        print(p.name, p.stat().st_size)


if __name__ == "__main__":
    main()
