"""Drop-in native operator fronts (core, dense, think, moe) over libkoemi_b200.so."""
