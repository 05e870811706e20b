"""Tensor-core and tensor-memory rates on this GPU (one CTA, clock64 cycles).

The decode attention kernel issues ``kind::f16`` MMAs of M = 128, K = 16 and N = 32 (the
24 query rows of a 4-token verify at 6:1 GQA) and writes its fp16 operands into TMEM with
``tcgen05.st``; its structure follows from these two rates:

* cycles per MMA by N, by the A operand's location (TMEM or shared memory) and by the
  number of independent accumulators the instructions rotate over;
* bytes per cycle of ``tcgen05.st.32x32b`` by storing warps and store width.

    python -m oscar_b200.bench.tcgen05_rates
"""
from __future__ import annotations

import json

import torch

from ..ops._ext import ext


def main(argv=None):
    torch.cuda.init()
    e = ext()
    iters = 200
    for n in (32, 64, 128, 256):
        for a_smem in (0, 1):
            issue, total = e.mma_rate(a_smem, 1, n, iters)
            print(json.dumps({"probe": "mma", "M": 128, "N": n, "K": 16, "A": "smem" if a_smem else "tmem",
                              "chains": 1, "cycles_per_mma": round(total / (iters * 16), 1),
                              "macs_per_cycle": round(128 * n * 16 / (total / (iters * 16)), 1)}), flush=True)
    for chains in (2, 4, 8):
        issue, total = e.mma_rate(0, chains, 32, iters)
        print(json.dumps({"probe": "mma", "M": 128, "N": 32, "K": 16, "A": "tmem", "chains": chains,
                          "cycles_per_mma": round(total / (iters * 16), 1)}), flush=True)
    st_iters = 2000
    for nw, width in ((1, 32), (4, 32), (8, 32), (16, 32), (4, 16), (4, 64)):
        cyc = max(e.tmem_store_rate(nw, width, st_iters))
        by = nw * st_iters * 32 * width * 4
        print(json.dumps({"probe": "tmem_store", "warps": nw, "columns": width,
                          "cycles_per_store": round(cyc / st_iters, 1), "bytes_per_cycle": round(by / cyc, 1)}),
              flush=True)


if __name__ == "__main__":
    main()
