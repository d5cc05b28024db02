"""Model targets whose regions the bundles swap (the reference's models/
catalogue, random-initialised to BASELINE's configs)."""
