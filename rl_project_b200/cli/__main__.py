import sys

from rl_project_b200.cli.main import main

sys.exit(main())
