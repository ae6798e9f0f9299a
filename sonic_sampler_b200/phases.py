"""Per-phase timeline of one fused singular call, from the phase-stamp diagnostic build.

    python -m sonic_sampler_b200.phases [config2|config5] [--calls N]

The diagnostic build (`python -m sonic_sampler_b200.build --stamps`, compiled with
-DSONIC_PHASE_STAMPS into _lib/libsonic_b200_stamps.so) records, in every CTA of the singular
kernel, %globaltimer at its phase boundaries and each warp's clock cycles per activity. This
script runs the config through that build, one call at a time with the stamps cleared in
between (L2 flushed before each call), and prints for the median call:

- the CTA timeline: when CTAs enter, finish set-up, see their first chunk, end streaming,
  fold, write their list, take the ticket; when the last CTA of each row merges and selects;
- per-warp activity: cycles waiting for the ring, processing groups, absorbing queues,
  releasing stages, and the keys pushed.

All times are microseconds from the earliest CTA entry of the call. The stamps themselves
cost a few percent; compare phases, not the absolute total, with `bench.py`.
"""

from __future__ import annotations

import ctypes
import os
import statistics
import sys
from pathlib import Path

import numpy as np

from sonic_sampler_b200 import build

PS_ENTRY, PS_PDL, PS_SETUP, PS_FIRST, PS_WARP0_END, PS_ALL_END, PS_FOLD, PS_LIST, PS_TICKET, PS_MERGE, PS_SELECT, \
    PS_SMID, PS_SCALARS, PS_ISSUED, PS_CTA_SLOTS = range(15)
PW_WAIT, PW_PROCESS, PW_ABSORB, PW_ABSORBS, PW_PUSHED, PW_RELEASE, PW_END, PW_GROUPS, PW_PUSHPATH, PW_LOADS, \
    PW_SLOTS = range(11)
PS_CTAS, NW = 8192, 8
CTA_BYTES = PS_CTAS * PS_CTA_SLOTS * 8
TOTAL_BYTES = CTA_BYTES + PS_CTAS * NW * PW_SLOTS * 8


def _library():
    path = build.build(stamps=True)
    os.environ["SONIC_B200_LIBRARY"] = str(path)
    from sonic_sampler_b200 import _abi

    lib = _abi.load_library()
    lib.sonic_phase_stamps.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32]
    lib.sonic_phase_stamps.restype = ctypes.c_int32
    return lib


def _read(lib) -> tuple[np.ndarray, np.ndarray]:
    buf = np.zeros(TOTAL_BYTES // 8, dtype=np.uint64)
    status = lib.sonic_phase_stamps(buf.ctypes.data, TOTAL_BYTES, 1)
    if status:
        raise RuntimeError(lib.sonic_last_error().decode())
    cta = buf[: PS_CTAS * PS_CTA_SLOTS].reshape(PS_CTAS, PS_CTA_SLOTS)
    warp = buf[PS_CTAS * PS_CTA_SLOTS:].reshape(PS_CTAS, NW, PW_SLOTS)
    return cta, warp


def _pct(x: np.ndarray) -> str:
    if x.size == 0:
        return "-"
    return f"{np.min(x):7.2f} {np.median(x):7.2f} {np.max(x):7.2f}"


def summarize(cta: np.ndarray, warp: np.ndarray, n_ctas: int, splits: int, clock_mhz: float) -> dict:
    cta = cta[:n_ctas].astype(np.int64)
    warp = warp[:n_ctas].astype(np.int64)
    t0 = cta[:, PS_ENTRY].min()
    rel = lambda col: (cta[:, col][cta[:, col] > 0] - t0) / 1e3  # noqa: E731 (us)
    lines = {}
    names = {PS_ENTRY: "entry", PS_PDL: "pdl wait done", PS_SCALARS: "slot scalars loaded",
             PS_ISSUED: "first chunks issued", PS_SETUP: "set-up done", PS_FIRST: "first chunk",
             PS_WARP0_END: "warp 0 streamed", PS_FOLD: "fold done", PS_LIST: "list written",
             PS_TICKET: "ticket", PS_MERGE: "row merge (last CTA)", PS_SELECT: "selection (last CTA)"}
    for col, name in names.items():
        lines[name] = _pct(rel(col))
    ends = warp[:, :, PW_END]
    warp_end = (ends[ends > 0] - t0) / 1e3
    lines["warp streamed+absorbed"] = _pct(warp_end)
    # per-CTA spread between its first and last warp
    spread = [(e[e > 0].max() - e[e > 0].min()) / 1e3 for e in ends if (e > 0).sum() > 1]
    lines["warp end spread in a CTA"] = _pct(np.array(spread))
    cyc = lambda i: warp[:, :, i].reshape(-1) / clock_mhz  # noqa: E731 (us)
    act = {"wait": cyc(PW_WAIT), "stage loads": cyc(PW_LOADS), "process": cyc(PW_PROCESS),
           "  of which push path": cyc(PW_PUSHPATH), "  of which absorb": cyc(PW_ABSORB), "release": cyc(PW_RELEASE)}
    per_warp = {k: _pct(v) for k, v in act.items()}
    per_warp["absorbs"] = _pct(warp[:, :, PW_ABSORBS].reshape(-1).astype(float))
    per_warp["keys pushed"] = _pct(warp[:, :, PW_PUSHED].reshape(-1).astype(float))
    per_warp["groups"] = _pct(warp[:, :, PW_GROUPS].reshape(-1).astype(float))
    sel = rel(PS_SELECT)
    sms = np.bincount(cta[:, PS_SMID], minlength=148)
    return {"timeline": lines, "per_warp": per_warp, "end_us": float(sel.max()) if sel.size else float("nan"),
            "ctas_per_sm": {int(k): int(v) for k, v in zip(*np.unique(sms, return_counts=True))}}


def main(argv: list[str]) -> None:
    import torch

    from sonic_sampler_b200 import workloads

    name = argv[0] if argv and not argv[0].startswith("--") else "config2"
    calls = int(argv[argv.index("--calls") + 1]) if "--calls" in argv else 5
    lib = _library()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if name == "config2":
        from sonic_sampler_b200.interface import UnshardedFusedSingular

        sets = [workloads.config2(dev, seed=1000 + 97 * i) for i in range(4)]
        sampler = UnshardedFusedSingular.initialize(128256, batch_size=64)
        run = lambda i: sampler.autoregressive(sets[i % 4]["logits"], sets[i % 4]["buffers"], logprobs=True)  # noqa
        rows, vocab = 64, 128256
    else:
        fn = workloads.runner(name, dev)
        run = lambda i: fn()  # noqa: E731
        rows, vocab = (1024, 256000) if name == "config5" else (64, 128256)
    a = __import__("sonic_sampler_b200._abi", fromlist=["SingularArgs"]).SingularArgs()
    a.rows, a.vocab_size = rows, vocab
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    for i in range(3):
        run(i)
    torch.cuda.synchronize()
    splits = None
    results, raw = [], []
    save = argv[argv.index("--save") + 1] if "--save" in argv else None
    for i in range(calls):
        _read(lib)  # clears
        flush.fill_(i & 0xFF)
        torch.cuda.synchronize()
        run(i)
        torch.cuda.synchronize()
        cta, warp = _read(lib)
        n = int((cta[:, PS_ENTRY] > 0).sum())
        results.append(summarize(cta, warp, n, splits, clock_mhz=_clock_mhz()))
        raw.append((cta[:n].copy(), warp[:n].copy()))
    order = sorted(range(calls), key=lambda i: results[i]["end_us"])
    med = results[order[calls // 2]]
    if save:
        c, w = raw[order[calls // 2]]
        np.savez(save, cta=c, warp=w)
    print(f"{name}: {calls} calls, median call (last selection at {med['end_us']:.2f} us after the first CTA entry)")
    print(f"CTAs per SM (count of SMs): {med['ctas_per_sm']}")
    print(f"{'CTA phase (us from first entry)':34s}   min  median     max")
    for k, v in med["timeline"].items():
        print(f"  {k:32s} {v}")
    print(f"{'per-warp activity (us of clock)':34s}   min  median     max")
    for k, v in med["per_warp"].items():
        print(f"  {k:32s} {v}")


def _clock_mhz() -> float:
    try:
        import subprocess

        out = subprocess.run(["nvidia-smi", "--id=0", "--query-gpu=clocks.sm", "--format=csv,noheader,nounits"],
                             capture_output=True, text=True, timeout=10).stdout.strip()
        return float(out.splitlines()[0])
    except Exception:
        return 1965.0


if __name__ == "__main__":
    main(sys.argv[1:])
