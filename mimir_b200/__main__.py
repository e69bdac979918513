from mimir_b200.cli import main

main()
