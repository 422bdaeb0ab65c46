/* Forced include for the reference build: include/generic.hpp uses
 * uint32_t without including <cstdint>. */
#pragma once
#include <cstdint>
