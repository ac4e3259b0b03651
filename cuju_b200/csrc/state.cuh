// cuju-b200: the per-environment match state.
//
// The content is fixed by GRF's serialized engine state (the bytes of `get_state`), so every
// member below is a field of that format; `io(A&)` visits them in the format's order for the host
// codec (codec.cpp). The reference declares the same schema in
// cuju include/cuju/state/environment_state.h:52-853; the field set and order must be identical
// for byte-compatible states. The device keeps one `Match` per environment in HBM, and the per-tick
// working set is cached by the SM's L1/L2.
#pragma once

#include "geom.cuh"

namespace cb {

constexpr int kTeamPlayers = 11;
constexpr int kPlayers = 2 * kTeamPlayers;
constexpr int kBodyParts = 14;
constexpr int kNodes = 14;
constexpr int kAnimPositions = 320;
constexpr int kControllers = 32;
constexpr int kMatchKeyboards = 22;
constexpr int kTactics = 14;

// GRF's radian: `angle - pi` when `rotated`. Stored with its 3 padding bytes.
struct Radian {
    float angle;
    bool rotated;
    uint8_t pad[3];
    CB_HD float value() const { return rotated ? angle - kPi : angle; }
};
static_assert(sizeof(Radian) == 8, "radian");
CB_HD void set_radian(Radian &r, float v) { r.angle = v; r.rotated = false; }

// A fixed-capacity list stored as a count and its elements.
template <class T, int N>
struct FVec {
    static constexpr int kCap = N;
    int32_t count;
    T el[N];
    CB_HD T &operator[](int i) { return el[i]; }
    CB_HD const T &operator[](int i) const { return el[i]; }
};

// Visitor tags the codec interprets.
enum PtrKind { kPtrPlayer, kPtrTeam, kPtrGamer, kPtrKeyboard, kPtrAnimation };

struct BiasedOffset {
    Quat orientation;
    float bias;
    template <class A> void io(A &a) { a.f(orientation); a.f(bias); }
};
struct MovementHistoryEntry {
    Vec3 position;
    Quat orientation;
    int32_t timeDiff_ms;
    int32_t nodeName;
    template <class A> void io(A &a) { a.f(position); a.f(orientation); a.f(timeDiff_ms); a.f(nodeName); }
};
struct NodeState {
    Vec3 position;
    Quat rotation;
    Vec3 scale;
    int32_t localMode;
    template <class A> void io(A &a) { a.f(position); a.f(rotation); a.f(scale); a.f(localMode); }
};
struct TouchInfo {
    Vec3 inputDirection;
    float inputPower, autoDirectionBias, autoPowerBias;
    Vec3 desiredDirection;
    float desiredPower;
    int32_t targetPlayer, forcedTargetPlayer;
    template <class A> void io(A &a) {
        a.f(inputDirection); a.f(inputPower); a.f(autoDirectionBias); a.f(autoPowerBias);
        a.f(desiredDirection); a.f(desiredPower); a.p(targetPlayer, kPtrPlayer);
        a.p(forcedTargetPlayer, kPtrPlayer);
    }
};
struct PlayerCommand {
    int32_t desiredFunctionType;
    bool useDesiredMovement;
    Vec3 desiredDirection;
    int32_t strictMovement;
    float desiredVelocityFloat;
    bool useDesiredLookAt;
    Vec3 desiredLookAt;
    bool useTouchInfo;
    TouchInfo touchInfo;
    bool onlyDeflectAnimationsThatPickupBall, useTripType;
    int32_t tripType;
    bool useDesiredTripDirection;
    Vec3 desiredTripDirection;
    bool useSpecialVar1;
    int32_t specialVar1;
    bool useSpecialVar2;
    int32_t specialVar2;
    int32_t modifier;
    template <class A> void io(A &a) {
        a.f(desiredFunctionType); a.f(useDesiredMovement); a.f(desiredDirection);
        a.f(strictMovement); a.f(desiredVelocityFloat); a.f(useDesiredLookAt);
        a.f(desiredLookAt); a.f(useTouchInfo); touchInfo.io(a);
        a.f(onlyDeflectAnimationsThatPickupBall); a.f(useTripType); a.f(tripType);
        a.f(useDesiredTripDirection); a.f(desiredTripDirection); a.f(useSpecialVar1);
        a.f(specialVar1); a.f(useSpecialVar2); a.f(specialVar2); a.f(modifier);
    }
};
struct FormationEntry {
    int32_t role;
    Vec3 position, startPosition;
    bool lazy, controllable;
    template <class A> void io(A &a) { a.f(role); a.f(position); a.f(startPosition); a.f(lazy); a.f(controllable); }
};
struct PlayerImage {
    Vec3 position, directionVector, movement;
    int32_t player;
    int32_t velocity, role;
    template <class A> void io(A &a) {
        a.f(position); a.f(directionVector); a.f(movement); a.p(player, kPtrPlayer);
        a.f(velocity); a.f(role);
    }
};
struct RotationSmuggle {
    Radian begin, end;
    template <class A> void io(A &a) { a.f(begin); a.f(end); }
};
struct AnimationState {
    int32_t anim;
    int32_t id, frameNumber, functionType, originatingInterrupt;
    Vec3 actionSmuggle, actionSmuggleOffset, actionSmuggleSustain, actionSmuggleSustainOffset,
        movementSmuggle, movementSmuggleOffset;
    RotationSmuggle rotationSmuggle;
    Radian rotationSmuggleOffset;
    int32_t touchFrame;
    Vec3 touchPosition, incomingMovement, outgoingMovement, positionOffset;
    PlayerCommand originatingCommand;
    FVec<Vec3, kAnimPositions> positions;
    template <class A> void io(A &a) {
        a.p(anim, kPtrAnimation); a.f(id); a.f(frameNumber); a.f(functionType);
        a.f(originatingInterrupt); a.f(actionSmuggle); a.f(actionSmuggleOffset);
        a.f(actionSmuggleSustain); a.f(actionSmuggleSustainOffset); a.f(movementSmuggle);
        a.f(movementSmuggleOffset); rotationSmuggle.io(a); a.f(rotationSmuggleOffset);
        a.f(touchFrame); a.f(touchPosition); a.f(incomingMovement); a.f(outgoingMovement);
        a.f(positionOffset); originatingCommand.io(a);
        a.vec(positions, [&](Vec3 &v) { a.f(v); });
    }
};
struct ApplyBuffer {
    int32_t anim;
    int32_t frameNumber;
    bool smooth;
    float smoothFactor;
    bool noPosition;
    Vec3 position;
    Radian orientation;
    BiasedOffset offsets[kBodyParts];
    template <class A> void io(A &a) {
        a.p(anim, kPtrAnimation); a.f(frameNumber); a.f(smooth); a.f(smoothFactor);
        a.f(noPosition); a.f(position); a.f(orientation);
        for (int i = 0; i < kBodyParts; i++) offsets[i].io(a);
    }
};
struct SpatialState {
    Vec3 position;
    Radian angle;
    Vec3 directionVector;
    int32_t velocityCategory;
    float floatVelocity;
    Vec3 actualMovement, physicsMovement, animationMovement, movement, actionSmuggleMovement,
        movementSmuggleMovement, positionOffsetMovement;
    Radian bodyAngle;
    Vec3 bodyDirectionVector;
    Radian relBodyAngleNonQuantized, relBodyAngle;
    Vec3 relBodyDirectionVector, relBodyDirectionVectorNonQuantized;
    int32_t foot;
    template <class A> void io(A &a) {
        a.f(position); a.f(angle); a.f(directionVector); a.f(velocityCategory); a.f(floatVelocity);
        a.f(actualMovement); a.f(physicsMovement); a.f(animationMovement); a.f(movement);
        a.f(actionSmuggleMovement); a.f(movementSmuggleMovement); a.f(positionOffsetMovement);
        a.f(bodyAngle); a.f(bodyDirectionVector); a.f(relBodyAngleNonQuantized);
        a.f(relBodyAngle); a.f(relBodyDirectionVector); a.f(relBodyDirectionVectorNonQuantized);
        a.f(foot);
    }
};
struct Humanoid {
    NodeState nodes[kNodes];
    ApplyBuffer applyBuffer;
    BiasedOffset offsets[kBodyParts];
    AnimationState anim;
    int32_t prevAnimFrameNumber, prevAnimFunctionType;
    Vec3 startPosition;
    Radian startAngle;
    Vec3 nextStartPosition;
    Radian nextStartAngle;
    SpatialState spatial;
    Vec3 previousPosition2D;
    int32_t interruptAnim, requeueDelayFrames, tripType;
    Vec3 tripDirection, decayingPositionOffset;
    float decayingDifficultyFactor;
    FVec<MovementHistoryEntry, 32> movementHistory;
    int32_t mentalImageTime;
    template <class A> void io(A &a) {
        for (int i = 0; i < kNodes; i++) nodes[i].io(a);
        applyBuffer.io(a);
        for (int i = 0; i < kBodyParts; i++) offsets[i].io(a);
        anim.io(a);
        a.f(prevAnimFrameNumber); a.f(prevAnimFunctionType); a.f(startPosition);
        a.f(startAngle); a.f(nextStartPosition); a.f(nextStartAngle); spatial.io(a);
        a.f(previousPosition2D); a.f(interruptAnim); a.f(requeueDelayFrames); a.f(tripType);
        a.f(tripDirection); a.f(decayingPositionOffset); a.f(decayingDifficultyFactor);
        a.vec(movementHistory, [&](MovementHistoryEntry &e) { e.io(a); });
        a.f(mentalImageTime);
    }
};
struct ControllerState {
    int32_t player;
    Vec3 inputDirection;
    float inputVelocityFloat;
    int32_t team, opponentTeam;
    int32_t opponentPlayer;
    float timeNeeded_ms;
    int32_t mentalImageTime;
    uint64_t lastSwitchTime_ms;
    uint32_t lastSwitchTimeDuration_ms;
    bool hasPossession, hasUniquePossession, teamHasPossession, teamHasUniquePossession,
        oppTeamHasPossession, oppTeamHasUniquePossession, hasBestPossession, teamHasBestPossession;
    float possessionAmount, teamPossessionAmount, fadingTeamPossessionAmount;
    int32_t oppTimeNeededToGetToBall;
    bool hasBestChanceOfPossession;
    template <class A> void io(A &a) {
        a.p(player, kPtrPlayer); a.f(inputDirection); a.f(inputVelocityFloat);
        a.p(team, kPtrTeam); a.p(opponentTeam, kPtrTeam); a.p(opponentPlayer, kPtrPlayer);
        a.f(timeNeeded_ms); a.f(mentalImageTime); a.f(lastSwitchTime_ms);
        a.f(lastSwitchTimeDuration_ms); a.f(hasPossession); a.f(hasUniquePossession);
        a.f(teamHasPossession); a.f(teamHasUniquePossession); a.f(oppTeamHasPossession);
        a.f(oppTeamHasUniquePossession); a.f(hasBestPossession); a.f(teamHasBestPossession);
        a.f(possessionAmount); a.f(teamPossessionAmount); a.f(fadingTeamPossessionAmount);
        a.f(oppTimeNeededToGetToBall); a.f(hasBestChanceOfPossession);
    }
};
struct AIControllerState {
    ControllerState base;
    bool ballBoundForGoal;
    float ballBoundForGoalY;
    Vec3 lastDesiredDirection;
    float lastDesiredVelocity;
    template <class A> void io(A &a) {
        base.io(a); a.f(ballBoundForGoal); a.f(ballBoundForGoalY); a.f(lastDesiredDirection);
        a.f(lastDesiredVelocity);
    }
};
struct Keyboard {
    float mirror;  // the stored direction is the true one times `mirror` (1 or -1)
    Vec3 direction;
    bool disabled;
    bool buttons[11];
    template <class A> void io(A &a) {
        a.f(mirror); a.f(direction); a.f(disabled);
        for (int i = 0; i < 11; i++) a.f(buttons[i]);
    }
};
struct HumanControllerState {
    ControllerState base;
    Keyboard keyboard;
    int32_t actionMode, actionButton, actionBufferTime_ms, gauge_ms;
    Vec3 previousDirection, steadyDirection;
    int32_t lastSteadyDirectionSnapshotTime_ms;
    template <class A> void io(A &a) {
        base.io(a); keyboard.io(a); a.f(actionMode); a.f(actionButton);
        a.f(actionBufferTime_ms); a.f(gauge_ms); a.f(previousDirection); a.f(steadyDirection);
        a.f(lastSteadyDirectionSnapshotTime_ms);
    }
};
struct HumanGamer {
    int32_t selectedPlayer;
    int32_t team;
    int32_t keyboardIndex;
    HumanControllerState controller;
    template <class A> void io(A &a) {
        a.p(selectedPlayer, kPtrPlayer); a.p(team, kPtrTeam); a.p(keyboardIndex, kPtrKeyboard);
        controller.io(a);
    }
};
struct NoController {
    template <class A> void io(A &) {}
};
template <class C>
struct PersonBase {
    bool isActive;
    Humanoid humanoid;
    C controller;
    int32_t externalController;
    uint64_t lastTouchTime_ms;
    int32_t lastTouchType;
    float fatigueFactorInverse;
    FVec<Vec3, 512> positionHistoryPerSecond;
    template <class A> void io(A &a) {
        a.f(isActive);
        humanoid.io(a);
        // GRF stores the controller of an active person only.
        if (isActive) controller.io(a);
        a.p(externalController, kPtrGamer); a.f(lastTouchTime_ms); a.f(lastTouchType);
        a.f(fatigueFactorInverse);
        a.vec(positionHistoryPerSecond, [&](Vec3 &v) { a.f(v); });
    }
};
struct TacticalSituation {
    float forwardSpaceRating, toGoalSpaceRating, spaceRating, forwardRating;
    template <class A> void io(A &a) {
        a.f(forwardSpaceRating); a.f(toGoalSpaceRating); a.f(spaceRating); a.f(forwardRating);
    }
};
struct Player {
    PersonBase<AIControllerState> base;
    int32_t manMarking;
    FormationEntry dynamicFormationEntry;
    bool hasPossession, hasBestPossession, hasUniquePossession;
    int32_t possessionDuration_ms;
    uint32_t timeNeededToGetToBall_ms, timeNeededToGetToBallOptimistic_ms,
        timeNeededToGetToBallPrevious_ms;
    bool triggerControlledBallCollision;
    TacticalSituation tactical;
    bool bufferNameCaptionShowCondition;
    Vec3 bufferPlayerColor;
    int32_t desiredTimeToBall_ms, cards;
    uint64_t cardEffectiveTime_ms;
    template <class A> void io(A &a) {
        base.io(a); a.p(manMarking, kPtrPlayer); dynamicFormationEntry.io(a);
        a.f(hasPossession); a.f(hasBestPossession); a.f(hasUniquePossession);
        a.f(possessionDuration_ms); a.f(timeNeededToGetToBall_ms);
        a.f(timeNeededToGetToBallOptimistic_ms); a.f(timeNeededToGetToBallPrevious_ms);
        a.f(triggerControlledBallCollision); tactical.io(a); a.f(bufferNameCaptionShowCondition);
        a.f(bufferPlayerColor); a.f(desiredTimeToBall_ms); a.f(cards); a.f(cardEffectiveTime_ms);
    }
};

// The team tactics: GRF keeps a map from 14 keys to `%f` texts; the float of each text is kept
// with a presence bit. Keys in alphabetical order (the order GRF stores the map in).
enum Tactic {
    kDefenseDepth, kDefenseMicroFocusStrength, kDefenseMidfieldFocus, kDefenseMidfieldFocusStrength,
    kDefenseOwnHalf, kDefenseSideFocusStrength, kDefenseWidth, kOffenseDepth,
    kOffenseMicroFocusStrength, kOffenseMidfieldFocus, kOffenseMidfieldFocusStrength,
    kOffenseOwnHalf, kOffenseSideFocusStrength, kOffenseWidth
};
struct Tactics {
    uint32_t present;
    float value[kTactics];
    template <class A> void io(A &a) { a.tactics(*this); }
};
struct OpponentInfo {
    int32_t player;
    float dangerFactor;
    template <class A> void io(A &a) { a.p(player, kPtrPlayer); a.f(dangerFactor); }
};
struct TeamAIState {
    int32_t taker;
    int32_t setPieceType;
    Tactics baseTactics, liveTactics;
    float offensivenessBias;
    bool teamHasPossession, teamHasUniquePossession, oppTeamHasPossession,
        oppTeamHasUniquePossession, teamHasBestPossession;
    float teamPossessionAmount, fadingTeamPossessionAmount;
    int32_t timeNeededToGetToBall, oppTimeNeededToGetToBall;
    float depth, width, offsideTrapX;
    uint64_t endApplyAttackingRun_ms;
    int32_t attackingRunPlayer;
    uint64_t endApplyTeamPressure_ms;
    int32_t teamPressurePlayer;
    uint64_t endApplyKeeperRush_ms;
    int32_t forwardSupportPlayer;
    FVec<OpponentInfo, kTeamPlayers> opponentInfo;
    template <class A> void io(A &a) {
        a.p(taker, kPtrPlayer); a.f(setPieceType); baseTactics.io(a); liveTactics.io(a);
        a.f(offensivenessBias); a.f(teamHasPossession); a.f(teamHasUniquePossession);
        a.f(oppTeamHasPossession); a.f(oppTeamHasUniquePossession); a.f(teamHasBestPossession);
        a.f(teamPossessionAmount); a.f(fadingTeamPossessionAmount); a.f(timeNeededToGetToBall);
        a.f(oppTimeNeededToGetToBall); a.f(depth); a.f(width); a.f(offsideTrapX);
        a.f(endApplyAttackingRun_ms); a.p(attackingRunPlayer, kPtrPlayer);
        a.f(endApplyTeamPressure_ms); a.p(teamPressurePlayer, kPtrPlayer);
        a.f(endApplyKeeperRush_ms); a.p(forwardSupportPlayer, kPtrPlayer);
        a.vec(opponentInfo, [&](OpponentInfo &o) { o.io(a); });
    }
};
struct Team {
    bool hasPossession;
    int32_t timeNeededToGetToBall_ms;
    int32_t designatedTeamPossessionPlayer;
    float teamPossessionAmount, fadingTeamPossessionAmount;
    TeamAIState ai;
    FVec<HumanGamer, kTeamPlayers> gamers;
    FVec<int32_t, kTeamPlayers> switchPriority;
    int32_t lastTouchPlayer, mainSelectedPlayer;
    template <class A> void io(A &a) {
        a.f(hasPossession); a.f(timeNeededToGetToBall_ms);
        a.p(designatedTeamPossessionPlayer, kPtrPlayer); a.f(teamPossessionAmount);
        a.f(fadingTeamPossessionAmount); ai.io(a);
        a.vec(gamers, [&](HumanGamer &g) { g.io(a); });
        a.vec(switchPriority, [&](int32_t &p) { a.f(p); });
        a.p(lastTouchPlayer, kPtrPlayer); a.p(mainSelectedPlayer, kPtrPlayer);
    }
};
struct MentalImage {
    uint32_t timeStamp_ms;
    float maxDistanceDeviation, maxMovementDeviation;
    FVec<PlayerImage, kPlayers> players;
    FVec<Vec3, 320> ballPredictions;
    // Not in the state: the predictions hold negated x and y (applied when read).
    bool lazyFlip;
    template <class A> void io(A &a) {
        a.f(timeStamp_ms); a.f(maxDistanceDeviation); a.f(maxMovementDeviation);
        a.vec(players, [&](PlayerImage &p) { p.io(a); });
        a.vec(ballPredictions, [&](Vec3 &v) { a.f(v); });
    }
};
struct Ball {
    Vec3 momentum;
    Quat rotationPerMs;
    Vec3 predictions[401];
    int32_t validPredictions;
    Quat orientationPrediction;
    FVec<Vec3, 402> positionHistory;
    Vec3 positionBuffer;
    Quat orientationBuffer;
    bool touchesNet;
    // Not in the state: `predictions` and `positionHistory` hold negated x and y.
    bool lazyFlip;
    template <class A> void io(A &a) {
        a.f(momentum); a.f(rotationPerMs);
        for (int i = 0; i < 401; i++) a.f(predictions[i]);
        a.f(validPredictions); a.f(orientationPrediction);
        a.vec(positionHistory, [&](Vec3 &v) { a.f(v); });
        a.f(positionBuffer); a.f(orientationBuffer); a.f(touchesNet);
    }
};
struct RefereeBuffer {
    bool active;
    int32_t desiredSetPiece;
    int32_t teamID;
    int32_t setPieceTeam;
    uint64_t stopTime, prepareTime, startTime;
    Vec3 restartPosition;
    int32_t taker;
    bool endPhase;
    template <class A> void io(A &a) {
        a.f(active); a.f(desiredSetPiece); a.f(teamID); a.p(setPieceTeam, kPtrTeam);
        a.f(stopTime); a.f(prepareTime); a.f(startTime); a.f(restartPosition);
        a.p(taker, kPtrPlayer); a.f(endPhase);
    }
};
struct Foul {
    int32_t foulPlayer, foulVictim;
    int32_t foulType;
    bool advantage;
    uint64_t foulTime;
    Vec3 foulPosition;
    bool hasBeenProcessed;
    template <class A> void io(A &a) {
        a.p(foulPlayer, kPtrPlayer); a.p(foulVictim, kPtrPlayer); a.f(foulType); a.f(advantage);
        a.f(foulTime); a.f(foulPosition); a.f(hasBeenProcessed);
    }
};
struct Referee {
    RefereeBuffer buffer;
    int32_t afterSetPieceRelaxTime_ms;
    FVec<int32_t, kTeamPlayers> offsidePlayers;
    Foul foul;
    template <class A> void io(A &a) {
        buffer.io(a); a.f(afterSetPieceRelaxTime_ms);
        a.vec(offsidePlayers, [&](int32_t &p) { a.f(p); });
        foul.io(a);
    }
};
struct Scenario {
    Vec3 ballPosition;
    int32_t leftTeamSize, rightTeamSize, leftAgents, rightAgents;
    bool useMagnet, offsides;
    float leftTeamDifficulty, rightTeamDifficulty;
    bool deterministic, endEpisodeOnScore, endEpisodeOnPossessionChange, endEpisodeOnOutOfPlay;
    int32_t gameDuration, secondHalf;  // in steps
    bool controlAllPlayers;
    bool realTime;
    uint32_t gameEngineRandomSeed;
    bool reverseTeamProcessing;  // the teams swap sides
    FormationEntry leftTeam[kTeamPlayers], rightTeam[kTeamPlayers];
    template <class A> void io(A &a) {
        a.f(ballPosition); a.f(leftTeamSize); a.f(rightTeamSize);
        a.check_team_sizes(leftTeamSize, rightTeamSize);
        a.f(leftAgents); a.f(rightAgents); a.f(useMagnet);
        a.f(offsides); a.f(leftTeamDifficulty); a.f(rightTeamDifficulty); a.f(deterministic);
        a.f(endEpisodeOnScore); a.f(endEpisodeOnPossessionChange); a.f(endEpisodeOnOutOfPlay);
        a.f(gameDuration); a.f(secondHalf); a.f(controlAllPlayers); a.f(realTime);
        a.f(gameEngineRandomSeed); a.f(reverseTeamProcessing);
        for (int i = 0; i < leftTeamSize; i++) leftTeam[i].io(a);
        for (int i = 0; i < rightTeamSize; i++) rightTeam[i].io(a);
    }
};

struct MatchState {
    int32_t firstTeam, secondTeam;  // team indices stored first and second
    FVec<MentalImage, 4> mentalImages;
    Team teams[2];
    int32_t playerCount;  // not in the state
    Player players[kPlayers];
    int32_t goalCount[2];
    float possessionLastMinute;
    PersonBase<NoController> officials[3];  // referee, then the two linesmen
    Keyboard secondKeyboardCopies[kControllers];
    int32_t freeControllerCount;  // not in the state
    Keyboard freeControllers[kControllers];
    Ball ball;
    uint64_t matchTime_ms, actualTime_ms, goalScoredTimer;
    int32_t matchPhase;
    bool inPlay, inSetPiece, goalScored, ballIsInGoal;
    int32_t lastGoalTeam;
    int32_t lastGoalScorer;
    int32_t lastTouchTeamIDs[4];  // GRF team IDs, one per touch type
    int32_t lastTouchTeamID;
    int32_t bestPossessionTeam;
    int32_t designatedPossessionPlayer;
    int32_t ballRetainer;
    uint32_t possessionSideHistoryMaxTime_ms;
    FVec<float, 600> possessionSideHistory;
    bool autoUpdateInGameCamera;
    Quat cameraOrientation, cameraNodeOrientation;
    Vec3 cameraNodePosition;
    float cameraFieldOfView, cameraNearCap, cameraFarCap;
    FVec<Vec3, 160> cameraPosition;
    uint32_t lastBodyBallCollisionTime_ms;
    Referee referee;
};

// Frame bookkeeping that a state does not store: each team is mirrored for the call frame of the
// team being processed (cuju include/cuju/simulation/world.h:25-34).
struct FrameFlags {
    bool teamMirrored[2];
    int32_t teamSide[2];
    bool ballMirrored;
    bool humanoidMirrored[kPlayers];
    bool mentalBallMirrored[4];
};

// One environment's complete match: the serialized engine state plus frame bookkeeping.
struct Match {
    int32_t gameState;
    int32_t waitingForGameCount;
    uint8_t rng[2512];
    Scenario scenario;
    int32_t step;
    MatchState m;
    FrameFlags flags;
    int32_t playerTeamID[kPlayers];
    // 0: own formation entry; else 1 + the player whose entry is used (a sent-off keeper's heir).
    int8_t formationOverride[kPlayers];
    CB_HD int firstTeamID() const { return m.firstTeam ^ (scenario.reverseTeamProcessing ? 1 : 0); }
};

}  // namespace cb
