// (all binding groups are implemented in their own translation units)
