"""L0 utilities: interval algebra, JSON-over-TCP messaging, logging, serialisation."""
