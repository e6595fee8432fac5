"""Engine layer (cache engine, token database, memory, connectors, backends)."""
