"""python -m pegaflow_b200.compat <pegaflow package dir>: install the stand-in
for the compiled ``pegaflow.pegaflow`` extension into that package."""

import sys

from . import install

if __name__ == "__main__":
    if len(sys.argv) != 2:
        print(__doc__, file=sys.stderr)
        sys.exit(2)
    print(install(sys.argv[1]))
