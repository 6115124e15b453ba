"""Runs the reference's own probe kernels (built from the reference sources
for sm_100a by `make -C oracle ref-gpu` into oracle/_ref/ref_gpu) on a B200
and stores their outputs as fixtures that pin the oracle:

ref_gpu_fixtures.json
    init_stream_4099      kernel_init_stream (src/mem_global.cu:5-12), 4099 words
    chase_cg              kernel_random_chase_cg (src/memory_chase.cu:29-34) final
                          index on the link array orc_chase_build(4096 slots,
                          seed 0xC0DA) for three (warmup, iters) pairs
    stream_copy_1mib_identical   kernel_stream_copy output == input
    hmma_*_sum_iters1000  kernel_hmma_{bf16,int8}_throughput outputs (sum of a
                          thread's four accumulators after 1000 all-ones MMAs)

Run on a machine with a B200, with the binary built beforehand where the
reference sources are:
    python tests/golden/make_ref_fixtures.py OUT.json
and store OUT.json next to this script as ref_gpu_fixtures.json.
"""

import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CHASE_SLOTS, CHASE_SEED = 4096, 0xC0DA


def main(out_path: str) -> None:
    import numpy as np

    import oracle

    orc = oracle.load()
    links = np.empty(CHASE_SLOTS * 32, np.uint32)
    orc.orc_chase_build(oracle.ptr(links), links.nbytes, CHASE_SEED)
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_gpu")
    with tempfile.NamedTemporaryFile(suffix=".bin", delete=False) as f:
        f.write(links.tobytes())
        path = f.name
    subprocess.run([exe, "fixtures", path, out_path], check=True)
    os.unlink(path)
    print("wrote", out_path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "ref_gpu_fixtures.json"))
