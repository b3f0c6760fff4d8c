"""Per-CTA timeline of the decode kernel over 36 Qwen3-4B-shape layers at 32k
(config 3), for a measurement build of the library: compiled with
-DGKV_PROBE_TIMELINE, which records globaltimer stamps per CTA (start, ids
staged, consumers released, first stage, last stage, merge) and per stage
(when consumer warp 0 passes each stage's full barrier) into device arrays
read back by gkv_probe_read_timeline / gkv_probe_read_stages.

    make -C genllm_b200/csrc OUT=<dir>/libprobe.so OBJDIR=<dir>/obj \\
         NVFLAGS="-O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -lineinfo -Xcompiler -fPIC \\
                  --expt-relaxed-constexpr -DGKV_PROBE_TIMELINE"
    GKV_LIB=<dir>/libprobe.so python -m genllm_b200.timeline_probe
    GKV_LIB=<dir>/libprobe.so torchrun --nproc-per-node N -m genllm_b200.timeline_probe   # sharded

Prints, for the last 8 decode launches, min/median/max over the CTAs of each
stamp (us from the first CTA start), then one layer's stage-ready times
relative to its release. Under torchrun the KV heads are sharded over the
ranks and each layer runs the fused head all-gather; the combine rows then
add the gather's phases (peer stores done, flags published, peers' flags
seen), printed by every rank for its own GPU. The product build has none of
this.
"""
import ctypes as C
import os

import numpy as np
import torch

from genllm_b200 import _lib
from genllm_b200.workload import DecodeWorkload


def main():
    ctx = int(os.environ.get("CTX", "32768"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("gloo")
    wl = DecodeWorkload(local, n_layers=36, ctx=ctx, pool_pages=max(4096, ctx // 16 + 64), world=world, rank=rank)
    s = torch.cuda.current_stream()
    sh = C.c_void_p(s.cuda_stream)
    hg = None
    if world > 1:
        from genllm_b200.gather import HeadGather
        hg = HeadGather(local, 36, wl.Hq)
    for _ in range(6):
        for l in range(36):
            if hg is None:
                wl.layer_step(l, sh)
            else:
                b = wl.layers[l]
                hg.decode(wl.mgr, l, b.q, b.k, b.v, wl.scale)
    torch.cuda.synchronize()
    L = _lib.lib()
    n = 8 * 4096 * 8
    buf = (C.c_ulonglong * n)()
    L.gkv_probe_read_timeline.argtypes = [C.c_void_p, C.c_int]
    if L.gkv_probe_read_timeline(buf, n) != 0:
        raise RuntimeError("not a measurement build (GKV_PROBE_TIMELINE)")
    a = np.frombuffer(buf, dtype=np.uint64).reshape(8, 4096, 8).astype(np.int64)
    rows = []
    for slot in range(8):
        d, c = a[slot, :2048], a[slot, 2048:]
        dv, cv = d[d[:, 0] > 0], c[c[:, 0] > 0]
        rows.append((dv[:, 0].min(), slot, dv, cv))
    rows.sort()
    t0 = rows[0][0]

    def st(x):
        x = x[x > 0] - t0
        return f"{x.min() / 1e3:7.2f}/{np.median(x) / 1e3:7.2f}/{x.max() / 1e3:7.2f}" if len(x) else "-"

    print(f"rank {rank}: decode: start | ids | released | first stage | end | merge | exit ;; combine: start | "
          "after wait | store | stores+ticket | flags out | peers seen   (min/med/max us)")
    for _, slot, dv, cv in rows:
        print(f"D n={len(dv)} {st(dv[:, 0])} | {st(dv[:, 1])} | {st(dv[:, 5])} | {st(dv[:, 2])} | {st(dv[:, 3])} | "
              f"{st(dv[:, 7])} | {st(dv[:, 4])}")
        print(f"C n={len(cv)} {st(cv[:, 0])} | {st(cv[:, 1])} | {st(cv[:, 2])} | {st(cv[:, 3])} | {st(cv[:, 4])} | "
              f"{st(cv[:, 5])}")
    m = 8 * 2048 * 16
    sb = (C.c_ulonglong * m)()
    L.gkv_probe_read_stages.argtypes = [C.c_void_p, C.c_int]
    L.gkv_probe_read_stages(sb, m)
    sa = np.frombuffer(sb, dtype=np.uint64).reshape(8, 2048, 16).astype(np.int64)
    _, slot, dv, _ = rows[4]
    k = len(dv)
    rel = sa[slot, :k] - a[slot, :k, 5][:, None]
    print("stage-ready after release, one layer (us): stage: min med max")
    for i in range(16):
        x = rel[:, i][sa[slot, :k, i] > 0]
        if len(x):
            print(i, f"{x.min() / 1e3:6.2f} {np.median(x) / 1e3:6.2f} {x.max() / 1e3:6.2f}")
    if hg is not None:
        hg.close()


if __name__ == "__main__":
    main()
