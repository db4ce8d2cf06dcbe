import sys

from .server.cli import main

sys.exit(main())
