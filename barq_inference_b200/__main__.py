"""``python -m barq_inference_b200 <subcommand> ...`` — the ``barq-inference`` command line."""
import sys

from .cli import main

sys.exit(main())
