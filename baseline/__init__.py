"""Reference install (baseline/_ref) helpers: build recipe and module loader."""
