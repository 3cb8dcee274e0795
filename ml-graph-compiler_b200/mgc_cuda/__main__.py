"""``python -m mgc_cuda``: the reference's ``mgc`` command line with the cuda target."""

import sys

from mgc_cuda.cli import main

sys.exit(main())
