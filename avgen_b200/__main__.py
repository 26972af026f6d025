"""``python -m avgen_b200`` runs the command line."""
from avgen_b200.cli.main import main

raise SystemExit(main())
