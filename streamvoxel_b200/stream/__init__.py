"""Drop-in mirror of the reference's `streamvoxel.stream` hot path: conditions, slot engine, EASE slots, admission."""
