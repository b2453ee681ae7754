"""python -m diffusionhard_b200 <subcommand> ..."""

from .cli import main

raise SystemExit(main())
