"""CLI of the feature-production pipeline: ``python -m flare_b200.data.run --config pipeline.yaml``.

The config file (YAML or JSON) holds the ``PipelineConfig`` fields; dense and
sparse column specs are lists of mappings, e.g.::

    inputs: [logs/]
    output: features/
    feature_column: 2
    label_code: 1
    dense: [{code: 10, transform: log1p}]
    sparse: [{kind: hash, codes: [20], buckets: 1000000}, {kind: cross, codes: [20, 21], buckets: 100000}]

Reference behaviour: src/flare/data/run.py:172.
"""
from __future__ import annotations

import json
import sys

from ..config.loader import LayeredConfigLoader
from .pipeline import DataPipeline, PipelineConfig


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    workers = 1
    if "--workers" in argv:
        i = argv.index("--workers")
        workers = int(argv[i + 1])
        del argv[i:i + 2]
    cfg = LayeredConfigLoader().load(PipelineConfig, argv)
    man = DataPipeline(cfg).run(workers=workers)
    print(json.dumps({"windows": len(man["windows"]), "rows": sum(w["rows"] for w in man["windows"]),
                      "inputs": len(man["inputs_done"])}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
