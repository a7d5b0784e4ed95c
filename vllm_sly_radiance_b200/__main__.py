from .entrypoints.cli import main

main()
