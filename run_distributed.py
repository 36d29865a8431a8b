#!/usr/bin/env python
"""Multi-node runner entry point (``python run_distributed.py --role both --gpus 0,1 ...``).

Thin wrapper around :mod:`zeroq_b200.run_distributed`; run it with ``--help``
for the options.
"""

import sys

from zeroq_b200.run_distributed import main

if __name__ == "__main__":
    sys.exit(main())
