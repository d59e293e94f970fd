"""Reference arm of the benchmark: runs the unmodified reference package installed in baseline/_ref."""
