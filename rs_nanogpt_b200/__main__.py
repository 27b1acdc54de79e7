import os
import sys

from .cli import main

rc = main()
if os.environ.get("RS_NANOGPT_RANK") is not None:
    # A spawned rank leaves without interpreter teardown: communication
    # libraries' transport threads must not be destroyed while a peer may
    # still be closing its side.
    sys.stdout.flush()
    sys.stderr.flush()
    os._exit(rc)
sys.exit(rc)
