"""The reference's own GPU implementation recompiled for sm_100a (comparator; not product code)."""
