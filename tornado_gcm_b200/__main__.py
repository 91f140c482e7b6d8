"""``python -m tornado_gcm_b200`` runs the command-line interface."""

from tornado_gcm_b200.cli import main

main()
