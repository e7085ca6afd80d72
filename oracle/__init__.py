"""CPU oracle (test infrastructure only): see oracle.py and cpu_path.py."""
