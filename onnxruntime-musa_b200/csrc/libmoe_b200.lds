{
  global:
    moe_b200_*;
  local:
    *;
};
