"""``python -m flare_b200 {train,recipe,eval} ...``: the framework's command line (``flare_b200.cli``)."""
from .cli import main

if __name__ == "__main__":
    raise SystemExit(main())
