// cuju-b200: read-only tables that every environment of a batch shares: the animation tables
// parsed from `animations.bin` (plus values derived from them once on the host), the skeletons
// and static player data of each scenario variant. They sit in HBM once per GPU and stay L2
// resident; the kernels read them through `const __restrict__` pointers.
// Layouts follow the file formats (cuju include/cuju/animation/animation_data.h:20-121,
// skeleton.h:22-48, simulation/static_data.h:17-61).
#pragma once

#include "state.cuh"

namespace cb {

enum AnimString {  // GRF e_AnimationString
    kAS_Empty = 0, kAS_OutgoingSpecialState = 1, kAS_IncomingSpecialState = 2,
    kAS_SpecialVariable1 = 3, kAS_SpecialVariable2 = 4, kAS_Type = 5, kAS_Trap = 6,
    kAS_Deflect = 7, kAS_Interfere = 8, kAS_Trip = 9, kAS_ShortPass = 10, kAS_LongPass = 11,
    kAS_Shot = 12, kAS_Sliding = 13, kAS_Movement = 14, kAS_Special = 15, kAS_BallControl = 16,
    kAS_HighPass = 17, kAS_Catch = 18, kAS_OutgoingRetainState = 19, kAS_IncomingRetainState = 20
};
enum StateString { kSS_Empty = 0, kSS_LayBack, kSS_LayFront, kSS_LeftElbow, kSS_RightElbow };

struct KeyFrame {
    int32_t frame;
    Quat orientation;
    Vec3 position;
};
// The pose of a node at a frame, tabulated for frames 0..frameCount+1 with the same function
// that computes it, so a read equals a computation bit for bit.
struct InterpEntry {
    Quat orientation;
    Vec3 position;
    float angleZ;  // yaw from Quat::angles
};
struct NodeAnim {
    int32_t bodyPart;
    int32_t firstKey, keyCount;
    int32_t interpOffset, interpFrames;
};
struct FootballKey {
    int32_t frame;
    Quat orientation;
    Vec3 position;
    float power;
};
struct Anim {
    int32_t frameCount, currentFoot, animationType;
    Vec3 translation, incomingMovement;
    float incomingVelocity;
    Vec3 outgoingMovement, outgoingDirection, incomingBodyDirection, outgoingBodyDirection;
    float outgoingVelocity;
    Radian outgoingAngle, incomingBodyAngle, outgoingBodyAngle;
    int32_t outgoingFoot;
    float idleLevel;
    int32_t quadrantID;
    float specialVar1, specialVar2;
    bool lastDitch, baseAnimation, hasFootball, hasPositions;
    int32_t outgoingSpecialState, incomingRetainState, incomingSpecialState;
    int32_t firstNode, nodeCount;
    int32_t firstFootball, footballCount;
    int32_t firstPosition, positionCount;
};
struct Quadrant {
    int32_t id;
    Vec3 position;
    int32_t velocity;
    Radian angle;
};
// Values derived from the text variables of each animation and animation-only subexpressions
// of the selection (cuju include/cuju/animation/animation_derived.h:67-166).
struct AnimDerived {
    double priorityAbsolute;
    int32_t touchFrame;
    float animDifficultyFactor;
    bool tripTypeIsOne;
    int32_t tripTypeRounded;
    Vec3 bumpDirection, incomingBallDirection, ballDirection;
    float incomingMaxDeviation, outgoingMaxDeviation;
    bool outgoingRetainRaw;
    int32_t outgoingRetainRawValue, incomingRetainRawValue;
    int32_t outgoingRetainBodyPart, incomingRetainBodyPart;
    int32_t forcedFootWhich;
    bool touchFootLeft;
    int32_t touchType;
    float touchMaxPowerFactor, touchDifficultyFactor;
    Vec3 crudeOutDirectionRotated;
    float crudeTurnAngle, crudeInBodyFixAbsolute;
    Vec3 crudeOutBodyDirection;
    bool crudeInBallNonzero;
    Vec3 crudeInBallAdapted, crudeBallDirectionNormalized;
    // Per-animation terms of the selection (cuju select_animation.h:470-509).
    float incomingBodyAngles[6];
    float bodyTurnAngle;
    int32_t incomingBodyIndex;
    Vec3 preferredOutgoingDirection, preferredOutgoingMovement;
    float preferredOutgoingAngle, lookAngle;
    int32_t smoothedMovementOffset;  // into AnimTables::smoothed, -1 below two positions
    bool ballDirectionFinite;
};

constexpr int kFunctionTypeSlots = 16;

struct AnimTables {
    const Anim *anims;
    const AnimDerived *derived;
    const NodeAnim *nodes;
    const KeyFrame *keys;
    const InterpEntry *interp;
    const FootballKey *football;
    const Vec3 *positions;
    const Quadrant *quadrants;
    const int16_t *functionAnims;   // animations per function type, increasing
    const int32_t *functionOffsets; // kFunctionTypeSlots + 1
    const Vec3 *smoothed;           // CalculateMovementAtFrame(positions, frame, 1) per frame
    int32_t animCount, quadrantCount;
    Radian maxIncomingBallDirDeviation, maxOutgoingBallDirDeviation;
};

// Skeleton of a humanoid (scene graph in pre-order).
struct SkelGeometry {
    bool footOrLowerLeg;
    int32_t localMode;
    Vec3 position;
    Quat rotation;
    Vec3 scale;
    Vec3 bbMin, bbMax;  // mesh space
};
struct SkelNode {
    int32_t parent;
    int32_t localMode;
    Vec3 position;
    Quat rotation;
    Vec3 scale;
    int32_t geometryCount;
    SkelGeometry geometries[2];
};
struct Skeleton {
    int32_t nodeMap[kBodyParts];
    int32_t nodeCount;
    SkelNode nodes[kNodes];
};

constexpr int kStatistics = 22;
enum Statistic {
    kStPhysicalBalance, kStPhysicalReaction, kStPhysicalAcceleration, kStPhysicalVelocity,
    kStPhysicalStamina, kStPhysicalAgility, kStPhysicalShotPower, kStTechnicalStandingTackle,
    kStTechnicalSlidingTackle, kStTechnicalBallControl, kStTechnicalDribble,
    kStTechnicalShortPass, kStTechnicalHighPass, kStTechnicalHeader, kStTechnicalShot,
    kStTechnicalVolley, kStMentalCalmness, kStMentalWorkRate, kStMentalResilience,
    kStMentalDefensivePositioning, kStMentalOffensivePositioning, kStMentalVision
};
struct PlayerData {
    float statistics[kStatistics];
    float velocityStatistic;
    float height;
    int32_t skinColor;
};
struct StaticFormation {
    int32_t role;
    Vec3 position, startPosition;
    bool lazy, controllable;
};
constexpr int kStaticEntries = kPlayers + 3;
// Players in state order, then the referee and the two linesmen.
struct StaticData {
    int32_t count;
    PlayerData data[kStaticEntries];
    StaticFormation formation[kStaticEntries];
    float matchDurationFactor;
    int32_t stableID[kStaticEntries];
};

// Everything a step reads besides the match itself, for one scenario variant.
struct Context {
    const AnimTables *anim;
    const StaticData *staticData;
    const Skeleton *skeletons;  // players, then officials
    const float *cameraWeights; // may be null
    int32_t ticksPerStep;
};

}  // namespace cb
