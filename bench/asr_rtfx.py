"""ASR throughput benchmark entry point under the reference's name
(VideoLingo-user bench/asr_rtfx.py:334-404 reports real-time factors of its
ASR backends).  Here it runs the repository's bench.py: the config-4 chunk
pipeline (log-mel + 32 x fused add+LayerNorm & GELU per 30 s chunk) on 1..N
B200s, with the reference's CPU path timed on the same box, printing one
JSON line.  Every bench.py flag is accepted, e.g.

    python bench/asr_rtfx.py --steps 10 --warmup 3
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        bench/asr_rtfx.py --gpus 8
"""

from __future__ import annotations

import runpy
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent

if __name__ == "__main__":
    sys.argv[0] = str(ROOT / "bench.py")
    runpy.run_path(str(ROOT / "bench.py"), run_name="__main__")
